"""The index plugin half of the boundary: the B200 index adapters
(elips_b200/integration/B200Indexes.cpp) selected by make_b200_index from an
elips::Config (make_index's selection, IndexFactory.cpp:40-50, and
make_gpu_index's, GpuHybridIndex.cpp:14-39) and driven through the
reference's own interfaces, IndexPort (insert / remove / search),
GpuIndexPort (build_from_batch / search_batch / export_to_cpu_index /
import_from_cpu_index) and IndexTransferPort (export / import_snapshot). They
are compiled against the reference headers into oracle/_ref/
libelips_ref_b200.so and compared with the reference's CPU classes on the same
RecordIDs:

  * B200BruteForceIndex vs ExactIndex (ExactIndex.cpp:55-87): fp32 (3xTF32)
    identical rows except ties within 1e-5, fp16 / bf16 recall >= 0.99; the
    same after inserts and removes (compaction included); filtered search vs
    ExactIndex over the candidate subset;
  * B200QuantizedIndex vs ExactIndex with the same Quantizer: bit-exact;
  * B200IvfPqIndex vs GpuIVFPQIndex on a CPU port: the exported model after
    build_from_batch, after one-by-one inserts (the retraining schedule of
    IvfIndexState::maybe_retrain_after_growth) and after removes is identical,
    and search results are identical outside rerank-boundary ties.
Error behaviour: DimensionMismatch thrown by insert and search on a bad width
(ExactIndex.cpp:14-20); search returns {} and search_batch a GpuError when
the backend refuses the call (GpuBruteForceIndex.cpp:112,117)."""
import numpy as np
import pytest

import oracle as O
from oracle import parity
from tests import helpers as H

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not O.REF_B200_SO.exists(), reason="reference-on-B200 driver not built")]


def _exact_ref(metric, base):
    return O.RefExactIndex(metric, base)


def _fp32_check(metric, base, q, d, r, rd, rr):
    res = parity.fp32_exact(d, r, rd, rr, lambda qi, row: O.distance(metric, q[qi], base[row]),
                            atol=1e-5 if metric == "cosine" else 0.0)
    assert res["pass"], res


@pytest.mark.parametrize("metric", ["euclidean", "cosine", "dot_product"])
def test_brute_force_index_matches_exact_index(metric):
    base = H.gaussian(3000, 48, seed=301)
    q = H.gaussian(64, 48, seed=302)
    if metric == "cosine":
        base, q = H.normalize(base), H.normalize(q)
    ix = O.B200PortIndex("brute_force", metric, 48, precision="fp32")
    assert ix.type_name().startswith("gpu_")
    assert ix.insert(base)
    assert ix.size() == 3000 and ix.device_bytes() > 0
    ref = _exact_ref(metric, base)
    d, r, bad = ix.search(q, 10)
    assert not bad
    rd, rr = ref.search(q, 10, 4)
    _fp32_check(metric, base, q, d, r, rd, rr)
    st, d2, r2 = ix.search_batch(q, 10)
    assert st == 0 and np.array_equal(r2, r) and np.array_equal(d2, d)


def test_brute_force_insert_remove_sequence_matches_exact_index():
    base = H.gaussian(2000, 32, seed=303)
    q = H.gaussian(40, 32, seed=304)
    ix = O.B200PortIndex("brute_force", "euclidean", 32, precision="fp32")
    ref = O.RefExactIndex("euclidean", base[:1000])
    assert ix.insert(base[:1000])
    ix.insert(base[1000:], first=1000)
    ref.insert(base[1000:], 1000)
    rng = np.random.default_rng(305)
    gone = rng.permutation(2000)[:1200]          # more than half: the device index compacts
    for step, row in enumerate(gone):
        ix.remove(int(row))
        ref.remove(int(row))
        if step in (10, 600, 1199):
            assert ix.size() == ref.size()
            d, r, _ = ix.search(q, 15)
            rd, rr = ref.search(q, 15, 4)
            _fp32_check("euclidean", base, q, d, r, rd, rr)
    ix.remove(5_000_000)                         # unknown id: no-op
    assert ix.size() == 800


@pytest.mark.parametrize("precision", ["fp16", "bf16"])
def test_brute_force_half_precision_recall(precision):
    cents = H.gaussian(64, 128, seed=306)
    base = H.mixture(20_000, 128, cents, 0.1, seed=307, normalized=True)
    q = H.mixture(100, 128, cents, 0.1, seed=308, normalized=True)
    ix = O.B200PortIndex("brute_force", "cosine", 128, precision=precision)
    ix.insert(base)
    st, d, r = ix.search_batch(q, 20)
    assert st == 0
    rounded = H.round_fp16(base) if precision == "fp16" else H.round_bf16(base)
    qr = H.round_fp16(q) if precision == "fp16" else H.round_bf16(q)
    rd, rr = O.exact_search("cosine", rounded, qr, 20)
    res = parity.low_precision(d, r, rd, rr)
    assert res["pass"], res


def test_brute_force_filtered_search_matches_candidate_subset():
    base = H.gaussian(5000, 64, seed=309)
    q = H.gaussian(30, 64, seed=310)
    cand = np.sort(np.random.default_rng(311).permutation(5000)[:500]).astype(np.int64)
    ix = O.B200PortIndex("brute_force", "euclidean", 64, precision="fp32")
    ix.insert(base)
    st, d, r = ix.search_batch(q, 10, candidates=cand)
    assert st == 0 and np.isin(r, cand).all()
    ref = O.RefExactIndex("euclidean", base[cand])
    rd, rr = ref.search(q, 10, 4)
    rr = cand[rr]
    _fp32_check("euclidean", base, q, d, r, rd, rr)
    st, d, r = ix.search_batch(q, 10, candidates=np.zeros(0, np.int64))   # empty candidate set: nothing
    assert st == 0 and (r == -1).all()


def test_brute_force_errors_follow_the_reference():
    base = H.gaussian(200, 16, seed=312)
    ix = O.B200PortIndex("brute_force", "euclidean", 16)
    assert not ix.insert(base[:, :15])                       # DimensionMismatch on insert
    assert ix.size() == 0
    ix.insert(base)
    _, _, bad = ix.search(H.gaussian(2, 17, seed=313), 5)     # DimensionMismatch on search
    assert bad
    # the library refuses k > 1024: search returns {} (no hits), search_batch a GpuError
    big = O.B200PortIndex("brute_force", "euclidean", 16)
    big.insert(H.gaussian(3000, 16, seed=314))
    d, r, bad = big.search(base[:2], 2000)
    assert not bad and (r == -1).all()
    st, _, _ = big.search_batch(base[:2], 2000)
    assert st != 0


def test_brute_force_snapshots_and_cpu_transfer():
    base = H.gaussian(1500, 24, seed=315)
    q = H.gaussian(20, 24, seed=316)
    a = O.B200PortIndex("brute_force", "euclidean", 24)
    a.insert(base)
    for row in range(0, 1500, 7):
        a.remove(row)
    b = O.B200PortIndex("brute_force", "euclidean", 24)
    assert a.copy_snapshot_to(b) == 0 and b.size() == a.size()
    d1, r1, _ = a.search(q, 12)
    d2, r2, _ = b.search(q, 12)
    assert np.array_equal(r1, r2) and np.array_equal(d1, d2)
    # export_to_cpu_index: the CPU ExactIndex now answers like the reference's own
    cpu = a.export_to_cpu("euclidean")
    keep = np.array([i for i in range(1500) if i % 7], np.int64)
    ref = O.RefExactIndex("euclidean", base[keep])
    cd, cr = cpu.search(q, 12, 4)
    rd, rr = ref.search(q, 12, 4)
    assert np.array_equal(cr, keep[rr]) and np.array_equal(cd, rd)
    # import_from_cpu_index back into a fresh device index
    c = O.B200PortIndex("brute_force", "euclidean", 24)
    assert c.import_from_cpu(cpu) == 0
    d3, r3, _ = c.search(q, 12)
    assert np.array_equal(r3, r1) and np.array_equal(d3, d1)


@pytest.mark.parametrize("codec", ["sq8", "pq"])
def test_quantized_index_bit_exact(codec):
    base = H.gaussian(4000, 32, seed=317)
    q = H.gaussian(25, 32, seed=318)
    if codec == "sq8":
        mins, scales = O.ref_sq8_train("euclidean", base)
        ix = O.B200PortIndex("quantized", "euclidean", 32, codec="sq8", params=np.concatenate([mins, scales]))
        ref = O.RefExactIndex("euclidean", base, codec="sq8", mins=mins, scales=scales)
    else:
        cb = O.ref_train_pq_codebook(base, 8, 64, 4)
        ix = O.B200PortIndex("quantized", "euclidean", 32, codec="pq", pq_dim=8, pq_bits=6, params=cb)
        ref = O.RefExactIndex("euclidean", base, codec="pq", codebook=cb, pq_bits=6)
    assert ix.type_name().startswith("gpu_")
    ix.insert(base)
    for row in (0, 17, 3999):
        ix.remove(row)
        ref.remove(row)
    d, r, _ = ix.search(q, 10)
    rd, rr = ref.search(q, 10, 4)
    assert np.array_equal(r, rr) and np.array_equal(d, rd)


def _ivf_model_data():
    cents = H.gaussian(64, 32, seed=320)
    base = H.mixture(12_000, 32, cents, 0.3, seed=321)
    q = H.mixture(60, 32, cents, 0.3, seed=322)
    return base, q


def test_ivfpq_build_from_batch_matches_reference():
    base, q = _ivf_model_data()
    cfg = dict(n_lists=64, nprobe=8, pq_dim=8, pq_bits=8, kmeans_iters=4)
    ix = O.B200PortIndex("ivf_pq", "euclidean", 32, **cfg)
    assert ix.build(base) == 0
    ref = O.RefIvfPqEmpty("euclidean", 32, **cfg)
    assert ref.build(base) == 0
    a = ix.export(len(base), 8, 256)
    b = ref.export(len(base), 8, 256)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)
    _, rows, asg, cb, codes = b
    cent = ref.centroids(64)
    assert np.array_equal(ix.centroids(64), cent)
    st, d, r = ix.search_batch(q, 10)
    assert st == 0
    rd, rr = ref.search(q, 10, 4)
    _, _, gap = O.ivfpq_search("euclidean", cent, cb, codes, base, asg, q, 8, 10, 4, with_gap=True)
    diff = [i for i in range(len(q)) if not (np.array_equal(r[i], rr[i]) and np.array_equal(d[i], rd[i]))]
    assert all(gap[i] == 0 for i in diff), diff
    d1, r1, _ = ix.search(q, 10)
    assert np.array_equal(r1, r) and np.array_equal(d1, d)


def test_ivfpq_insert_and_remove_follow_the_reference_lifecycle():
    base, q = _ivf_model_data()
    base = base[:400]
    cfg = dict(n_lists=16, nprobe=4, pq_dim=4, pq_bits=4, kmeans_iters=3)
    ix = O.B200PortIndex("ivf_pq", "euclidean", 32, **cfg)
    ref = O.RefIvfPqEmpty("euclidean", 32, **cfg)
    for i in range(0, 400, 1):
        ix.insert(base[i:i + 1], first=i)
        ref.insert(base[i:i + 1], first=i)
    for row in (3, 399, 100, 7):
        ix.remove(row)
        ref.remove(row)
    n = ref.size()
    assert ix.size() == n == 396
    a = ix.export(n, 4, 16)
    b = ref.export(n, 4, 16)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)
    assert np.array_equal(ix.centroids(16), ref.centroids(16))
    st, d, r = ix.search_batch(q, 5)
    rd, rr = ref.search(q, 5, 4)
    _, vec, asg, cb, codes = b
    _, _, gap = O.ivfpq_search("euclidean", ref.centroids(16), cb, codes, vec, asg, q, 4, 5, 4, with_gap=True)
    rows_of = b[0]
    diff = [i for i in range(len(q)) if not (np.array_equal(r[i], rr[i]) and np.array_equal(d[i], rd[i]))]
    assert st == 0 and all(gap[i] == 0 for i in diff), diff
