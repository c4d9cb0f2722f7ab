"""Incremental insert / remove and device snapshots of the exact index
(through the C ABI), against the oracle on the reference's semantics:

* GpuBruteForceIndex::remove erases the row and keeps the others in order
  (src/gpu_engine/GpuBruteForceIndex.cpp:84-99); insert appends
  (:77-82). The device index keeps a removed row's number reserved (a
  removal bit), so its results are the oracle's on the erased base mapped
  through the kept rows' numbers; after compact() the numbers are the
  erased base's own.
* IndexSnapshot round trip (IndexSnapshot.hpp:26-56): an imported index
  answers exactly as the exported one, removal bits included.

int8 (bit-exact scores, ties by row) makes every comparison exact; duplicate
rows make ties common, so the order of the surviving rows is exercised too."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _int8_rows(n, d, seed, distinct=None):
    rng = np.random.default_rng(seed)
    if distinct is None:
        return rng.integers(-127, 128, size=(n, d), dtype=np.int8)
    uniq = rng.integers(-3, 4, size=(distinct, d), dtype=np.int8)
    return uniq[rng.integers(0, distinct, size=n)]


def _index(base):
    from elips_b200 import ExactIndex
    ix = ExactIndex("dot_product", base.shape[1], precision="int8")
    ix.add(base)
    return ix


def _expected(base, live, queries, k):
    """Oracle on the erased base, rows mapped back to the original numbers."""
    kept = np.flatnonzero(live)
    d, r = O.int8_ip_search(base[kept], queries, k)
    return d, np.where(r >= 0, kept[np.maximum(r, 0)], -1)


@pytest.mark.parametrize("distinct", [None, 40])
def test_remove_matches_erased_reference(distinct):
    base = _int8_rows(12000, 96, seed=1, distinct=distinct)
    q = _int8_rows(60, 96, seed=2, distinct=distinct)
    ix = _index(base)
    live = np.ones(len(base), bool)
    rng = np.random.default_rng(3)
    for batch in (1, 37, 2000):
        for s in rng.choice(np.flatnonzero(live), batch, replace=False):
            assert ix.remove(int(s))
            live[s] = False
        d, r = ix.search_batch(q, 25)
        de, re_ = _expected(base, live, q, 25)
        assert np.array_equal(d, de) and np.array_equal(r, re_)
    assert ix.live() == live.sum() and ix.size() == len(base)


def test_remove_twice_and_out_of_range():
    from elips_b200 import _capi
    ix = _index(_int8_rows(100, 32, seed=4))
    assert ix.remove(7) and not ix.remove(7)
    with pytest.raises(_capi.ElipsB200Error):
        ix.remove(100)


def test_insert_after_remove_then_compact():
    base = _int8_rows(5000, 64, seed=5, distinct=30)
    more = _int8_rows(3000, 64, seed=6, distinct=30)
    q = _int8_rows(40, 64, seed=7, distinct=30)
    ix = _index(base)
    live = np.ones(len(base), bool)
    for s in range(0, 5000, 3):
        ix.remove(s)
        live[s] = False
    ix.add(more)
    allrows = np.concatenate([base, more])
    live = np.concatenate([live, np.ones(len(more), bool)])
    d, r = ix.search_batch(q, 30)
    de, re_ = _expected(allrows, live, q, 30)
    assert np.array_equal(d, de) and np.array_equal(r, re_)
    new_to_old = ix.compact()
    assert np.array_equal(new_to_old, np.flatnonzero(live))
    assert ix.size() == ix.live() == live.sum()
    d2, r2 = ix.search_batch(q, 30)
    dc, rc = O.int8_ip_search(allrows[live], q, 30)
    assert np.array_equal(d2, dc) and np.array_equal(r2, rc)


def test_remove_every_row():
    base = _int8_rows(300, 32, seed=8)
    ix = _index(base)
    for s in range(300):
        ix.remove(s)
    d, r = ix.search_batch(base[:3], 5)
    assert (r == -1).all() and np.isinf(d).all()
    assert ix.compact().shape == (0,) and ix.size() == 0


@pytest.mark.parametrize("precision,metric", [("int8", "dot_product"), ("fp32", "euclidean"),
                                              ("fp16", "cosine"), ("bf16", "euclidean")])
def test_snapshot_round_trip(precision, metric):
    from elips_b200 import ExactIndex
    rng = np.random.default_rng(9)
    if precision == "int8":
        base, q = _int8_rows(7000, 80, seed=10), _int8_rows(50, 80, seed=11)
    else:
        base = rng.standard_normal((7000, 80)).astype(np.float32)
        q = rng.standard_normal((50, 80)).astype(np.float32)
    a = ExactIndex(metric, 80, precision=precision)
    a.add(base)
    for s in range(0, 7000, 11):
        a.remove(s)
    blob = a.export_snapshot()
    b = ExactIndex(metric, 80, precision=precision)
    b.import_snapshot(blob)
    assert b.size() == a.size() and b.live() == a.live()
    da, ra = a.search_batch(q, 20)
    db, rb = b.search_batch(q, 20)
    assert np.array_equal(ra, rb) and np.array_equal(da, db)
    assert not np.isin(rb, np.arange(0, 7000, 11)).any()


def test_snapshot_rejects_other_shapes():
    from elips_b200 import ExactIndex, _capi
    a = ExactIndex("euclidean", 16, precision="fp16")
    a.add(np.ones((10, 16), np.float32))
    blob = a.export_snapshot()
    for metric, dim, prec in [("cosine", 16, "fp16"), ("euclidean", 32, "fp16"), ("euclidean", 16, "bf16")]:
        with pytest.raises(_capi.ElipsB200Error):
            ExactIndex(metric, dim, precision=prec).import_snapshot(blob)
    full = ExactIndex("euclidean", 16, precision="fp16")
    full.add(np.ones((1, 16), np.float32))
    with pytest.raises(_capi.ElipsB200Error):
        full.import_snapshot(blob)
    with pytest.raises(_capi.ElipsB200Error):
        ExactIndex("euclidean", 16, precision="fp16").import_snapshot(blob[:-8])


def test_ivfpq_snapshot_round_trip():
    """IVF-PQ snapshot readback equals what was imported (codes encoded on the
    device equal the oracle's encode_pq of the residuals), and an index rebuilt
    from it answers identically."""
    from elips_b200.ivfpq import IvfFlatIndex, IvfPqIndex
    from tests import helpers as H
    m = H.ivfpq_tie_model()
    base, q, cent, cb = m["base"], m["queries"][:60], m["cent"], m["cb"]
    asg = m["asg"]
    a = IvfPqIndex("euclidean", base.shape[1], cent, cb, nprobe=8)
    a.add(base, asg)
    snap = a.export_snapshot()
    assert np.array_equal(snap["centroids"], cent) and np.array_equal(snap["codebook"], cb)
    assert np.array_equal(snap["vectors"], base) and np.array_equal(snap["assignments"], asg)
    res = (base - cent[asg]).astype(np.float32)
    assert np.array_equal(snap["codes"], O.encode_pq(cb, res))
    b = IvfPqIndex("euclidean", base.shape[1], snap["centroids"], snap["codebook"], nprobe=8)
    b.add(snap["vectors"], snap["assignments"], snap["codes"])
    da, ra = a.search_batch(q, 10)
    db, rb = b.search_batch(q, 10)
    assert np.array_equal(ra, rb) and np.array_equal(da, db)
    f = IvfFlatIndex("euclidean", base.shape[1], cent, nprobe=8)
    f.add(base, asg)
    fs = f.export_snapshot()
    assert np.array_equal(fs["vectors"], base) and np.array_equal(fs["assignments"], asg)
    assert np.array_equal(fs["centroids"], cent)


def test_ivfpq_remove_and_rebuild_match_reference():
    """IVF-PQ remove + rebuild_codes against the reference's own
    GpuIVFPQIndex::remove (IvfIndexState::remove, then rebuild_codes) on the
    same imported snapshot: after the same removals the exported snapshots
    agree field by field, bit for bit (row order, vectors, lists, the
    retrained codebook and every code), and the searches return the same rows."""
    from elips_b200.ivfpq import IvfPqIndex
    from tests import helpers as H
    m = H.ivfpq_tie_model()
    n = 12000
    base, cent, cb = m["base"][:n], m["cent"], m["cb"]
    asg, codes = m["asg"][:n], m["codes"][:n]
    pq_dim, ksub = cb.shape[0], cb.shape[1]
    a = IvfPqIndex("euclidean", base.shape[1], cent, cb, nprobe=8)
    a.add(base, asg, codes)
    ref = O.RefIvfPqIndex("euclidean", cent, asg, cb, codes, base, 8)
    ids = list(range(n))  # slot -> original row, with the reference's swap
    for row in (5, n - 1, 17, 3000, 42, 11998):
        slot = ids.index(row)
        a.remove(slot)
        ref.remove(row)
        if slot != len(ids) - 1:
            ids[slot] = ids[-1]
        ids.pop()
    a.rebuild_codes()
    snap = a.export_snapshot()
    rrows, rvec, rasg, rcb, rcodes = ref.export(len(ids), pq_dim, ksub)
    assert np.array_equal(rrows, np.array(ids))
    assert np.array_equal(snap["vectors"], rvec) and np.array_equal(snap["assignments"], rasg)
    assert np.array_equal(snap["codebook"].view(np.uint32), rcb.view(np.uint32))
    assert np.array_equal(snap["codes"], rcodes)
    q = m["queries"][:50]
    d, r = a.search_batch(q, 10)
    d_ref, r_ref = ref.search(q, 10, 4)
    ids_arr = np.array(ids)
    mapped = np.where(r >= 0, ids_arr[np.maximum(r, 0)], -1)
    agree = np.mean([np.array_equal(mapped[i], r_ref[i]) for i in range(len(q))])
    assert agree >= 0.9, agree   # differences only where the rerank boundary is an exact tie
