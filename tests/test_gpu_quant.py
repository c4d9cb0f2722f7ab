"""Bit-exact parity of the SIMT paths (through the C ABI) with the oracle,
itself pinned to the reference:

  * GpuPort::compute_distances_batch / top_k (GpuPort.hpp:65-82);
  * ExactIndex + ProductQuantizer (plain and OPQ) and + ScalarQuantizer (sq8):
    codes, distances and slots identical to the reference's arithmetic.
"""
import numpy as np
import pytest

import oracle as O
from tests import helpers as H

pytestmark = pytest.mark.gpu

METRICS = ["cosine", "euclidean", "dot_product"]


@pytest.mark.parametrize("metric", METRICS)
@pytest.mark.parametrize("d", [4, 37, 128])
def test_compute_distances_batch_bit_exact(metric, d):
    from elips_b200.quant import compute_distances_batch
    db = H.gaussian(700, d, seed=41)
    q = H.gaussian(19, d, seed=42)
    out = compute_distances_batch(q, db, metric)
    ref = np.array([[O.distance(metric, q[i], db[j]) for j in range(db.shape[0])] for i in range(q.shape[0])],
                   np.float32)
    assert np.array_equal(out, ref)


def test_compute_distances_device_pointers_match_host():
    import torch
    from elips_b200 import _capi
    from elips_b200.quant import compute_distances_batch
    db = H.gaussian(3000, 64, seed=43)
    q = H.gaussian(40, 64, seed=44)
    host = compute_distances_batch(q, db, "euclidean")
    dq, ddb = torch.from_numpy(q).cuda(), torch.from_numpy(db).cuda()
    out = torch.empty((40, 3000), dtype=torch.float32, device="cuda")
    _capi.check(_capi.LIB.elips_b200_compute_distances_batch(0, dq.data_ptr(), ddb.data_ptr(), out.data_ptr(), 40,
                                                             3000, 64, 1, 1,
                                                             torch.cuda.current_stream().cuda_stream), "dist")
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), host)


@pytest.mark.parametrize("nb,k", [(10, 3), (5000, 64), (300, 1000), (70_000, 17), (5000, 4000), (3000, 5000), (200_000, 1500)])
def test_top_k_matches_stable_sort(nb, k):
    from elips_b200.quant import top_k
    rng = np.random.default_rng(45)
    d = rng.integers(0, 50, size=(7, nb)).astype(np.float32)  # many ties
    idx, val = top_k(d, k)
    order = np.argsort(d, axis=1, kind="stable")
    take = min(k, nb)
    assert np.array_equal(idx[:, :take], order[:, :take].astype(np.uint32))
    assert np.array_equal(val[:, :take], np.take_along_axis(d, order[:, :take], axis=1))
    if k > nb:
        assert (idx[:, nb:] == 0xFFFFFFFF).all() and np.isinf(val[:, nb:]).all()


@pytest.mark.parametrize("k", [20, 100, 400])
def test_top_k_never_takes_inf_or_nan(k):
    """Values of +inf and NaN are never among the k best (the warp-per-row
    kernel for k <= 256 and the block kernel above it agree): the finite
    values in stable order, then {0xFFFFFFFF, +inf} padding."""
    from elips_b200.quant import top_k
    rng = np.random.default_rng(46)
    d = rng.integers(0, 30, size=(9, 500)).astype(np.float32)
    d[rng.random(d.shape) < 0.6] = np.inf
    d[rng.random(d.shape) < 0.05] = np.nan
    d[:, :3] = -np.inf
    idx, val = top_k(d, k)
    for r in range(d.shape[0]):
        fin = np.flatnonzero(d[r] < np.inf)
        order = fin[np.argsort(d[r, fin], kind="stable")][:k]
        t = order.size
        assert np.array_equal(idx[r, :t], order.astype(np.uint32))
        assert np.array_equal(val[r, :t], d[r, order])
        assert (idx[r, t:] == 0xFFFFFFFF).all() and np.isposinf(val[r, t:]).all()


@pytest.fixture(scope="module")
def pq_data():
    base = H.gaussian(20_000, 64, seed=46)
    q = H.gaussian(150, 64, seed=47)
    return base, q


@pytest.mark.parametrize("metric", METRICS)
@pytest.mark.parametrize("bits", [8, 4])
def test_pq_search_bit_exact(metric, bits, pq_data, nthreads):
    from elips_b200.quant import QuantizedIndex
    base, q = pq_data
    cb = O.ref_train_pq_codebook(base[:4000], 16, 1 << bits, 4)
    ix = QuantizedIndex("pq", metric, 64, codebook=cb, pq_bits=bits)
    ix.add(base)                                   # encoded on the device
    codes = O.encode_pq(cb, base)
    d_ref, r_ref = O.pq_search(metric, cb, codes, q, 50, nthreads=nthreads)
    d, r = ix.search_batch(q, 50)
    assert np.array_equal(d, d_ref)
    assert np.array_equal(r, r_ref)


def test_pq_encode_matches_reference(pq_data):
    from elips_b200.quant import QuantizedIndex
    import torch
    base, q = pq_data
    cb = O.ref_train_pq_codebook(base[:4000], 16, 256, 4)
    # codes added as codes and codes produced on the device must search identically
    a = QuantizedIndex("pq", "euclidean", 64, codebook=cb)
    a.add(base)
    b = QuantizedIndex("pq", "euclidean", 64, codebook=cb)
    b.add_codes(O.ref_encode_pq(cb, base))
    da, ra = a.search_batch(q, 30)
    db, rb = b.search_batch(q, 30)
    assert np.array_equal(da, db) and np.array_equal(ra, rb)


@pytest.mark.parametrize("metric", METRICS)
def test_opq_search_bit_exact(metric, nthreads):
    from elips_b200.quant import QuantizedIndex
    base = H.gaussian(8000, 32, seed=48)
    q = H.gaussian(60, 32, seed=49)
    rot, _ = np.linalg.qr(np.random.default_rng(50).standard_normal((32, 32)))
    rot = rot.astype(np.float32)
    rb = O.rotate_rows(rot, base)
    cb = O.ref_train_pq_codebook(rb[:3000], 8, 256, 4)
    ix = QuantizedIndex("opq", metric, 32, codebook=cb, rotation=rot)
    ix.add(base)
    d, r = ix.search_batch(q, 20)
    d_ref, r_ref = O.RefExactIndex(metric, base, codec="opq", codebook=cb, pq_bits=8, rotation=rot).search(
        q, 20, nthreads)
    assert np.array_equal(d, d_ref) and np.array_equal(r, r_ref)


@pytest.mark.parametrize("metric", METRICS)
@pytest.mark.parametrize("d", [128, 300])
def test_sq8_search_bit_exact(metric, d, nthreads):
    from elips_b200.quant import QuantizedIndex
    base = H.gaussian(12_000, d, seed=51)
    q = H.gaussian(40, d, seed=52)
    mins, scales = O.sq8_train(base[:5000])          # later rows fall outside: clamped
    ix = QuantizedIndex("sq8", metric, d, mins=mins, scales=scales)
    ix.add(base)
    codes = O.sq8_encode(mins, scales, base)
    d_ref, r_ref = O.sq8_search(metric, mins, scales, codes, q, 25, nthreads=nthreads)
    dist, rows = ix.search_batch(q, 25)
    assert np.array_equal(dist, d_ref)
    assert np.array_equal(rows, r_ref)


def test_sq8_matches_reference_exact_index(nthreads):
    from elips_b200.quant import QuantizedIndex
    base = H.gaussian(6000, 64, seed=53)
    q = H.gaussian(30, 64, seed=54)
    mins, scales = O.ref_sq8_train("dot_product", base)
    ix = QuantizedIndex("sq8", "dot_product", 64, mins=mins, scales=scales)
    ix.add(base)
    d_ref, r_ref = O.RefExactIndex("dot_product", base, codec="sq8", mins=mins, scales=scales).search(q, 15, nthreads)
    d, r = ix.search_batch(q, 15)
    assert np.array_equal(d, d_ref) and np.array_equal(r, r_ref)


def test_quantized_edge_cases():
    from elips_b200.quant import QuantizedIndex
    mins, scales = np.zeros(8, np.float32), np.ones(8, np.float32)
    ix = QuantizedIndex("sq8", "euclidean", 8, mins=mins, scales=scales)
    d, r = ix.search_batch(np.zeros((2, 8), np.float32), 4)
    assert (r == -1).all()
    ix.add(np.arange(24, dtype=np.float32).reshape(3, 8))
    d, r = ix.search_batch(np.zeros((1, 8), np.float32), 5)
    assert list(r[0, :3]) == [0, 1, 2] and (r[0, 3:] == -1).all()


@pytest.mark.parametrize("n,d", [(1, 1), (33, 768), (1000, 37), (70_001, 128)])
def test_normalize_rows_bit_exact(n, d):
    from elips_b200.quant import normalize_rows
    rng = np.random.default_rng(n + d)
    x = (rng.standard_normal((n, d)) * rng.uniform(1e-3, 1e3, (n, 1))).astype(np.float32)
    x[0] = 0.0
    got = normalize_rows(x)
    assert np.array_equal(got.view(np.uint32), O.normalize_rows(x).view(np.uint32))


@pytest.mark.parametrize("codec,metric", [("sq8", "euclidean"), ("pq", "cosine"), ("sq8", "dot_product")])
def test_row_sharded_quantized_equals_single_index(codec, metric):
    """Row sharding of the quantized ExactIndex (split_ids ranges,
    GpuDistributedIndex.cpp:12-22), ranks emulated on one GPU: every shard's
    k results become (distance, global row) pairs, the merge kernel keeps the
    k smallest by (distance, row); ids and distances equal one index over all
    rows bit for bit (duplicate rows make ties across shards)."""
    import torch
    from elips_b200 import merge_candidates_device
    from elips_b200.distributed import shard_candidates, shard_range
    from elips_b200.quant import QuantizedIndex
    base = H.gaussian(9000, 64, seed=57)
    base[4500:4600] = base[100:200]          # identical rows in different shards
    q = H.gaussian(50, 64, seed=58)
    if codec == "sq8":
        mins, scales = O.sq8_train(base[:5000])
        make = lambda: QuantizedIndex("sq8", metric, 64, mins=mins, scales=scales)
    else:
        cb = O.ref_train_pq_codebook(base[:4000], 16, 256, 4)
        make = lambda: QuantizedIndex("pq", metric, 64, codebook=cb)
    full = make()
    full.add(base)
    qd = torch.from_numpy(q).cuda()
    d_ref, r_ref = full.search_device(qd, 30)
    for world in (2, 3, 8):
        blocks = []
        for rank in range(world):
            lo, hi = shard_range(base.shape[0], rank, world)
            ix = make()
            ix.add(base[lo:hi])
            d, r = ix.search_device(qd, 30)
            blocks.append(shard_candidates(d, r, lo))
        d, r = merge_candidates_device(torch.stack(blocks), world, 30, "dot_product")
        torch.cuda.synchronize()
        assert torch.equal(r, r_ref), world
        assert torch.equal(d.view(torch.int32), d_ref.view(torch.int32)), world
