"""Parity of the fused tensor-core exact search (through the C ABI) with the
oracle (oracle/oracle.c, pinned to the reference's ExactIndex::search,
src/ExactIndex.cpp:55-87).

Tolerances are the ones the backend promises:
  * fp32 (3xTF32): identical slots except ties within 1e-5 relative;
    distances within 1e-5 relative;
  * fp16 / bf16: recall >= 0.99 against the oracle run on the same rounded
    values, distances within 1e-2 relative;
  * int8: bit-exact distances and slots (ties broken by slot).
"""
import numpy as np
import pytest

import oracle as O
from tests import helpers as H

pytestmark = pytest.mark.gpu


def _index(metric, base, precision, device=0):
    from elips_b200 import ExactIndex
    ix = ExactIndex(metric, base.shape[1], precision=precision, device=device)
    ix.add(base)
    return ix


def _true(metric, base, queries):
    return lambda q, r: O.distance(metric, queries[q], base[r])


@pytest.mark.parametrize("metric", ["euclidean", "cosine", "dot_product"])
def test_fp32_matches_oracle_l2_config_shape(metric, nthreads):
    # N=100,000 x d=128 i.i.d. N(0,1), k=10: the fp32 exact configuration's base,
    # with a seeded 300-query slice.
    base = H.gaussian(100_000, 128, seed=1)
    queries = H.gaussian(300, 128, seed=2)
    if metric == "cosine":
        base, queries = H.normalize(base), H.normalize(queries)
    ix = _index(metric, base, "fp32")
    d, r = ix.search_batch(queries, 10)
    dr, rr = O.exact_search(metric, base, queries, 10, nthreads=nthreads)
    # cosine distances of unrelated unit vectors sit near 1: compare absolutely there
    atol = 1e-5 if metric == "cosine" else 0.0
    H.assert_ranked_match(d, r, dr, rr, _true(metric, base, queries), rtol=1e-5, atol=atol)
    assert np.array_equal(r, rr) or H.recall(r, rr) > 0.995


def test_fp16_cosine_clustered_recall(nthreads):
    # Clustered unit vectors like the fp16 cosine configuration (d=768, sigma=0.1),
    # reduced to 40,000 rows; the oracle sees the same fp16-rounded values.
    d = 768
    cents = H.gaussian(256, d, seed=3)
    base = H.round_fp16(H.mixture(40_000, d, cents, 0.1, seed=4, normalized=True))
    queries = H.round_fp16(H.mixture(200, d, cents, 0.1, seed=5, normalized=True))
    ix = _index("cosine", base, "fp16")
    dist, rows = ix.search_batch(queries, 100)
    dr, rr = O.exact_search("cosine", base, queries, 100, nthreads=nthreads)
    assert H.recall(rows, rr) >= 0.99
    np.testing.assert_allclose(dist, dr, rtol=1e-2, atol=1e-4)
    assert (np.diff(dist, axis=1) >= 0).all()


@pytest.mark.parametrize("batch", [1, 8, 64])
def test_bf16_l2_filtered(batch, nthreads):
    # Filtered L2 over bf16 rows with a Bernoulli(0.1) eligibility mask, k=20.
    base = H.round_bf16(H.gaussian(60_000, 384, seed=6))
    queries = H.round_bf16(H.gaussian(batch, 384, seed=7))
    words, bits = H.bernoulli_mask(base.shape[0], 0.1, seed=8)
    ix = _index("euclidean", base, "bf16")
    dist, rows = ix.search_batch(queries, 20, mask=words)
    dr, rr = O.exact_search("euclidean", base, queries, 20, nthreads=nthreads, mask=words)
    assert bits[rows[rows >= 0]].all(), "a masked-out row was returned"
    assert H.recall(rows, rr) >= 0.99
    np.testing.assert_allclose(dist, dr, rtol=1e-2)


def test_int8_inner_product_bit_exact(nthreads):
    rng = np.random.default_rng(9)
    base = rng.integers(-127, 128, size=(30_000, 1024), dtype=np.int8)
    queries = rng.integers(-127, 128, size=(150, 1024), dtype=np.int8)
    ix = _index("dot_product", base, "int8")
    dist, rows = ix.search_batch(queries, 50)
    dr, rr = O.int8_ip_search(base, queries, 50, nthreads=nthreads)
    assert np.array_equal(dist, dr)
    assert np.array_equal(rows, rr)


def test_int8_ties_break_by_slot(nthreads):
    # Many duplicate rows: equal scores must come out in ascending slot order.
    rng = np.random.default_rng(10)
    uniq = rng.integers(-3, 4, size=(50, 64), dtype=np.int8)
    base = uniq[rng.integers(0, 50, size=4000)]
    queries = rng.integers(-3, 4, size=(20, 64), dtype=np.int8)
    ix = _index("dot_product", base, "int8")
    dist, rows = ix.search_batch(queries, 64)
    dr, rr = O.int8_ip_search(base, queries, 64, nthreads=nthreads)
    assert np.array_equal(dist, dr)
    assert np.array_equal(rows, rr)


@pytest.mark.parametrize("n,d,nq,k", [(1, 3, 1, 1), (7, 5, 3, 10), (300, 17, 129, 1),
                                      (5000, 200, 257, 1000), (20_000, 64, 2, 33)])
def test_fp32_edge_shapes(n, d, nq, k, nthreads):
    base = H.gaussian(n, d, seed=11)
    queries = H.gaussian(nq, d, seed=12)
    ix = _index("euclidean", base, "fp32")
    dist, rows = ix.search_batch(queries, k)
    dr, rr = O.exact_search("euclidean", base, queries, k, nthreads=nthreads)
    H.assert_ranked_match(dist, rows, dr, rr, _true("euclidean", base, queries), rtol=1e-5, atol=1e-6)
    if k > n:
        assert (rows[:, n:] == -1).all() and np.isinf(dist[:, n:]).all()


def test_empty_index_and_k_zero():
    from elips_b200 import ExactIndex
    ix = ExactIndex("euclidean", 4, precision="fp32")
    d, r = ix.search_batch(np.zeros((2, 4), np.float32), 3)
    assert (r == -1).all()
    d, r = ix.search_batch(np.zeros((2, 4), np.float32), 0)
    assert d.shape == (2, 0)


def test_all_rows_masked_out():
    base = H.gaussian(1000, 32, seed=13)
    ix = _index("euclidean", base, "fp16")
    words = np.zeros(32, np.uint32)
    d, r = ix.search_batch(base[:4], 5, mask=words)
    assert (r == -1).all()


def test_dimension_mismatch_raises():
    from elips_b200 import DimensionMismatch
    base = H.gaussian(10, 8, seed=14)
    ix = _index("euclidean", base, "fp32")
    with pytest.raises(DimensionMismatch):
        ix.search_batch(np.zeros((1, 9), np.float32), 1)


def test_incremental_add_matches_single_add(nthreads):
    base = H.gaussian(9000, 96, seed=15)
    queries = H.gaussian(40, 96, seed=16)
    from elips_b200 import ExactIndex
    ix = ExactIndex("euclidean", 96, precision="fp16")
    for chunk in np.array_split(base, 7):
        ix.add(chunk)
    assert ix.size() == base.shape[0]
    d1, r1 = ix.search_batch(queries, 25)
    d2, r2 = _index("euclidean", base, "fp16").search_batch(queries, 25)
    assert np.array_equal(r1, r2) and np.array_equal(d1, d2)


def test_reference_known_answers():
    # metrics_test.cpp:24-35 and GpuAdvancedIndexTest.cpp sample vectors.
    from elips_b200 import ExactIndex
    ix = ExactIndex("euclidean", 2, precision="fp32")
    ix.add(np.array([[3.0, 4.0]], np.float32))
    (slot, dist), = ix.search(np.array([0.0, 0.0], np.float32), 1)
    assert slot == 0 and abs(dist - 5.0) < 1e-6
    ix = ExactIndex("dot_product", 3, precision="fp32")
    ix.add(np.array([[1.0, 1.0, 1.0]], np.float32))
    (slot, dist), = ix.search(np.array([1.0, 2.0, 3.0], np.float32), 1)
    assert abs(dist + 6.0) < 1e-6
    sample = np.array([[0, 0, 0, 0], [0.1, 0.1, 0, 0], [5, 5, 5, 5], [5.2, 5.1, 5, 5],
                       [-4, -4, -4, -4], [-4.1, -4, -4, -4]], np.float32)
    ix = ExactIndex("euclidean", 4, precision="fp32")
    ix.add(sample)
    assert ix.search(np.array([-4.1, -4.0, -4.0, -4.0], np.float32), 2)[0][0] == 5
    assert ix.search(np.array([0.1, 0.1, 0.0, 0.0], np.float32), 1)[0][0] == 1


def test_device_api_matches_host_api():
    import torch
    base = H.gaussian(20_000, 128, seed=17)
    queries = H.gaussian(300, 128, seed=18)
    ix = _index("euclidean", base, "bf16")
    d1, r1 = ix.search_batch(queries, 16)
    qd = torch.from_numpy(queries).cuda()
    d2, r2 = ix.search_device(qd, 16)
    torch.cuda.synchronize()
    assert np.array_equal(d1, d2.cpu().numpy()) and np.array_equal(r1, r2.cpu().numpy())


def test_shard_candidates_merge_equals_single_index():
    # Row sharding as GpuDistributedIndex does (contiguous split_ids ranges,
    # GpuDistributedIndex.cpp:12-22), merged by the final top-k kernel.
    import torch
    from elips_b200 import merge_candidates_device
    base = H.gaussian(30_000, 64, seed=19)
    queries = H.gaussian(100, 64, seed=20)
    k = 40
    full = _index("euclidean", base, "fp32")
    d_ref, r_ref = full.search_batch(queries, k)
    shards = 3
    qd = torch.from_numpy(queries).cuda()
    cand = torch.empty((shards, 100, k, 2), dtype=torch.int32, device="cuda")
    for s in range(shards):
        lo, hi = base.shape[0] * s // shards, base.shape[0] * (s + 1) // shards
        ix = _index("euclidean", base[lo:hi], "fp32")
        ix.search_candidates_device(qd, k, lo, cand[s])
    d, r = merge_candidates_device(cand, shards, k, "euclidean")
    torch.cuda.synchronize()
    assert np.array_equal(r.cpu().numpy(), r_ref)
    np.testing.assert_allclose(d.cpu().numpy(), d_ref, rtol=1e-6)


@pytest.mark.parametrize("precision,metric", [("fp16", "cosine"), ("int8", "dot_product"), ("fp32", "euclidean")])
def test_replicated_query_slices_equal_whole_batch(precision, metric):
    # Replicate mode (DistributedMode::replicate): each replica answers a
    # query_range slice of the batch; ranks emulated on one GPU. Slices of a
    # 300-query batch run the single-CTA kernel, the whole batch the CTA-pair
    # kernel: every query's results are identical either way.
    import torch
    from elips_b200.distributed import ReplicatedIndex, query_range
    rng = np.random.default_rng(23)
    if precision == "int8":
        base = rng.integers(-127, 128, size=(40_000, 96), dtype=np.int8)
        queries = rng.integers(-127, 128, size=(300, 96), dtype=np.int8)
    else:
        base = H.gaussian(40_000, 96, seed=24)
        queries = H.gaussian(300, 96, seed=25)
        if metric == "cosine":
            base, queries = H.normalize(base), H.normalize(queries)
    ix = _index(metric, base, precision)
    qd = torch.from_numpy(queries).cuda()
    d_ref, r_ref = ix.search_device(qd, 50)
    for world in (2, 3, 8):
        parts = [ix.search_device(qd[lo:hi], 50) for lo, hi in (query_range(300, r, world) for r in range(world))]
        assert torch.equal(torch.cat([p[1] for p in parts]), r_ref)
        assert torch.equal(torch.cat([p[0] for p in parts]).view(torch.int32), d_ref.view(torch.int32))
    one = ReplicatedIndex(ix)  # no process group: a single replica
    d1, r1 = one.search_device(qd, 50)
    assert one.world == 1 and one.size() == base.shape[0]
    assert torch.equal(r1, r_ref) and torch.equal(d1.view(torch.int32), d_ref.view(torch.int32))


@pytest.mark.parametrize("nq", [1300, 4000])
def test_int8_many_lists_two_stage_merge(nq):
    # Batches of a few thousand queries over a base cut into many splits give
    # each query more candidates (2 x splits x k) than the merge cache holds;
    # they are merged in two stages (groups of up to 16 lists, the last group
    # ragged). int8 scores are exact, ties by row: bit-identical to the oracle.
    rng = np.random.default_rng(29)
    base = rng.integers(-127, 128, size=(60_000, 64), dtype=np.int8)
    queries = rng.integers(-127, 128, size=(nq, 64), dtype=np.int8)
    ix = _index("dot_product", base, "int8")
    d, r = ix.search_batch(queries, 100)
    d_ref, r_ref = O.int8_ip_search(base, queries, 100)
    assert np.array_equal(r, r_ref) and np.array_equal(d, d_ref)


@pytest.mark.parametrize("shards", [2, 3])
def test_filtered_shards_merge_equals_single_index(shards):
    # Row-sharded filtered search, ranks emulated on one GPU: each shard gets
    # the global mask sliced to its rows (first row at bit 0); the merged
    # results equal one filtered index over all rows.
    import torch
    from elips_b200 import merge_candidates_device
    from elips_b200.distributed import shard_range, slice_mask
    base = H.gaussian(20_000, 48, seed=33)
    queries = H.gaussian(64, 48, seed=34)
    rng = np.random.default_rng(35)
    keep = rng.random(base.shape[0]) < 0.1
    words = np.zeros((base.shape[0] + 31) // 32, np.uint32)
    for i in np.flatnonzero(keep):
        words[i >> 5] |= np.uint32(1) << np.uint32(i & 31)
    k = 20
    full = _index("euclidean", base, "bf16")
    d_ref, r_ref = full.search_batch(queries, k, mask=words)
    assert keep[r_ref[r_ref >= 0]].all()
    qd = torch.from_numpy(queries).cuda()
    cand = torch.empty((shards, 64, k, 2), dtype=torch.int32, device="cuda")
    for s in range(shards):
        lo, hi = shard_range(base.shape[0], s, shards)
        ix = _index("euclidean", base[lo:hi], "bf16")
        m = torch.from_numpy(slice_mask(words, lo, hi).view(np.int32)).cuda()
        ix.search_candidates_device(qd, k, lo, cand[s], mask=m)
    d, r = merge_candidates_device(cand, shards, k, "euclidean")
    torch.cuda.synchronize()
    assert np.array_equal(r.cpu().numpy(), r_ref)
    np.testing.assert_allclose(d.cpu().numpy(), d_ref, rtol=1e-6)


def test_no_device_error_recorded():
    from elips_b200 import _capi
    assert _capi.device_error(0) == 0


@pytest.mark.parametrize("p,k", [(0.2, 10), (0.02, 50), (0.0, 5)])
def test_filtered_subset_gather_with_removals(p, k, nthreads):
    """A row filter selecting at most half of a large base is searched by
    gathering the selected live rows first; results (slots, distances) equal
    the oracle's scan restricted to filter AND live rows, ties by slot."""
    base = H.gaussian(100_000, 64, seed=41)
    base[50_000:50_100] = base[:100]                      # exact ties across the base
    queries = H.gaussian(150, 64, seed=42)
    words, bits = H.bernoulli_mask(base.shape[0], p, seed=43)
    ix = _index("euclidean", base, "fp32")
    removed = np.arange(7, 100_000, 997)
    for r in removed:
        ix.remove(int(r))
    live = np.ones(base.shape[0], bool)
    live[removed] = False
    dist, rows = ix.search_batch(queries, k, mask=words)
    sel = bits & live
    sel_words = np.zeros_like(words)
    idx = np.nonzero(sel)[0]
    np.bitwise_or.at(sel_words, idx >> 5, (np.uint32(1) << (idx & 31).astype(np.uint32)))
    dr, rr = O.exact_search("euclidean", base, queries, k, nthreads=nthreads, mask=sel_words)
    assert sel[rows[rows >= 0]].all()
    H.assert_ranked_match(dist, rows, dr, rr, _true("euclidean", base, queries), rtol=1e-5)
