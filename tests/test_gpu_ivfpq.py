"""IVF-PQ parity (through the C ABI) with the reference's GpuIVFPQIndex::search
(src/gpu_engine/GpuIVFPQIndex.cpp:161-237), run here from its own compiled
sources (oracle/_ref) and from the golden fixture it produced.

Returned ids and distances are the exact-reranked ones. The device path
chooses the R = max(4k, k) rows to rerank by (approximate distance, slot);
the reference uses std::partial_sort by distance alone, whose choice among
rows tied at the boundary is unspecified (rows with identical residual codes
in one list tie exactly). So: the device results equal the oracle's
device-order restatement on every query, and equal the reference's on every
query whose boundary is not tied; a query that differs from the reference
must have an exact tie at the boundary."""
from pathlib import Path

import numpy as np
import pytest

import oracle as O
from tests import helpers as H

pytestmark = pytest.mark.gpu


def test_ivfpq_golden_fixture():
    from elips_b200.ivfpq import IvfPqIndex
    G = np.load(Path(__file__).resolve().parent / "golden" / "reference_outputs.npz")
    ix = IvfPqIndex("euclidean", 24, G["ivf_centroids"], G["ivf_codebook"], nprobe=3, pq_bits=4)
    ix.add(G["base"], G["ivf_assignments"])          # residual codes encoded on the device
    assert np.array_equal(ix.codes(), G["ivf_codes"])
    d, r = ix.search_batch(G["queries"], 4)
    assert np.array_equal(r, G["ivf_rows"])
    assert np.array_equal(d, G["ivf_dist"])


@pytest.fixture(scope="module")
def model():
    return H.ivfpq_tie_model()


@pytest.mark.parametrize("nprobe,k", [(8, 10), (1, 5), (200, 3)])
def test_ivfpq_matches_reference(model, nprobe, k, nthreads):
    from elips_b200.ivfpq import IvfPqIndex
    m = model
    ix = IvfPqIndex("euclidean", 64, m["cent"], m["cb"], nprobe=nprobe)
    ix.add(m["base"], m["asg"], m["codes"])
    d, r = ix.search_batch(m["queries"], k)
    args = ("euclidean", m["cent"], m["cb"], m["codes"], m["base"], m["asg"], m["queries"], nprobe, k, nthreads)
    d_dev, r_dev = O.ivfpq_search(*args, order="device")
    assert np.array_equal(r, r_dev) and np.array_equal(d, d_dev)
    _, _, gap = O.ivfpq_search(*args, order="reference", with_gap=True)
    ref = O.RefIvfPqIndex("euclidean", m["cent"], m["asg"], m["cb"], m["codes"], m["base"], nprobe)
    d_ref, r_ref = ref.search(m["queries"], k, nthreads)
    differ = [q for q in range(r.shape[0]) if not (np.array_equal(r[q], r_ref[q]) and np.array_equal(d[q], d_ref[q]))]
    untied = [q for q in differ if gap[q] != 0]
    assert not untied, f"{len(untied)} queries without a boundary tie differ from the reference, first {untied[:5]}"


def test_ivfpq_device_codes_match_reference_encode(model):
    from elips_b200.ivfpq import IvfPqIndex
    m = model
    ix = IvfPqIndex("euclidean", 64, m["cent"], m["cb"], nprobe=8)
    ix.add(m["base"][:20_000], m["asg"][:20_000])
    ix.add(m["base"][20_000:], m["asg"][20_000:])
    assert np.array_equal(ix.codes(), m["codes"])


@pytest.mark.parametrize("metric", ["cosine", "dot_product"])
def test_ivfpq_inner_product_metrics_match_reference(metric, nthreads):
    from elips_b200.ivfpq import IvfPqIndex
    d, nlist = 32, 40
    base = H.normalize(H.gaussian(8000, d, seed=64))
    q = H.normalize(H.gaussian(50, d, seed=65))
    cent = O.ref_kmeans(base, nlist, 4)
    asg = O.ivf_assign(metric, base, cent)
    res = base - cent[asg]
    cb = O.ref_train_pq_codebook(res, 4, 64, 4)
    codes = O.ref_encode_pq(cb, res)
    ix = IvfPqIndex(metric, d, cent, cb, nprobe=6, pq_bits=6)
    ix.add(base, asg, codes)
    dist, rows = ix.search_batch(q, 7)
    d_dev, r_dev = O.ivfpq_search(metric, cent, cb, codes, base, asg, q, 6, 7, nthreads, order="device")
    assert np.array_equal(rows, r_dev) and np.array_equal(dist, d_dev)
    _, _, gap = O.ivfpq_search(metric, cent, cb, codes, base, asg, q, 6, 7, nthreads, with_gap=True)
    d_ref, r_ref = O.RefIvfPqIndex(metric, cent, asg, cb, codes, base, 6, pq_bits=6).search(q, 7, nthreads)
    differ = [i for i in range(len(q)) if not (np.array_equal(rows[i], r_ref[i]) and np.array_equal(dist[i], d_ref[i]))]
    assert all(gap[i] == 0 for i in differ)


def test_ivfpq_device_api_and_empty_index(model):
    import torch
    from elips_b200.ivfpq import IvfPqIndex
    m = model
    empty = IvfPqIndex("euclidean", 64, m["cent"], m["cb"], nprobe=4)
    d, r = empty.search_batch(m["queries"][:3], 5)
    assert (r == -1).all()
    ix = IvfPqIndex("euclidean", 64, m["cent"], m["cb"], nprobe=4)
    vd = torch.from_numpy(m["base"]).cuda()
    ad = torch.from_numpy(m["asg"].view(np.int32)).cuda()
    ix.add_device(vd, ad)
    d1, r1 = ix.search_batch(m["queries"], 10)
    d2, r2 = ix.search_device(torch.from_numpy(m["queries"]).cuda(), 10)
    torch.cuda.synchronize()
    assert np.array_equal(r1, r2.cpu().numpy()) and np.array_equal(d1, d2.cpu().numpy())


def test_ivfpq_rejects_bad_assignment(model):
    from elips_b200 import ElipsB200Error
    from elips_b200.ivfpq import IvfPqIndex
    m = model
    ix = IvfPqIndex("euclidean", 64, m["cent"], m["cb"], nprobe=4)
    bad = m["asg"][:10].copy()
    bad[3] = 128  # one past the last list
    with pytest.raises(ElipsB200Error):
        ix.add(m["base"][:10], bad)
    assert ix.size() == 0


@pytest.mark.parametrize("world,balanced", [(2, False), (3, False), (3, True)])
@pytest.mark.parametrize("metric", ["euclidean", "dot_product"])
def test_list_sharded_search_equals_single_index(model, world, balanced, metric):
    """List-sharded IVF-PQ (one rank per list range), its ranks driven phase by
    phase in one process on one GPU: the result equals the single index's."""
    import torch
    from elips_b200.distributed import ShardedIvfPqIndex
    from elips_b200.ivfpq import IvfPqIndex
    m = model
    base, q = m["base"], m["queries"]
    asg, codes = m["asg"], m["codes"]
    if metric != "euclidean":
        base, q = H.normalize(base), H.normalize(q)
        asg = O.ivf_assign(metric, base, m["cent"])
        codes = O.ref_encode_pq(m["cb"], base - m["cent"][asg])
    k, nprobe = 10, 8
    single = IvfPqIndex(metric, 64, m["cent"], m["cb"], nprobe=nprobe)
    single.add(base, asg, codes)
    d_ref, r_ref = single.search_batch(q, k)
    vd, ad, cd = (torch.from_numpy(base).cuda(), torch.from_numpy(asg.view(np.int32)).cuda(),
                  torch.from_numpy(codes).cuda())
    from elips_b200.distributed import balanced_lists
    owner = balanced_lists(np.bincount(asg, minlength=len(m["cent"])), world) if balanced else None
    ranks = [ShardedIvfPqIndex(metric, 64, m["cent"], m["cb"], nprobe, rank=r, world=world, owner=owner)
             for r in range(world)]
    for ix in ranks:
        for r0 in range(0, len(base), 25_000):  # rows offered in global order, in batches
            ix.add_device(vd[r0:r0 + 25_000], ad[r0:r0 + 25_000], r0, cd[r0:r0 + 25_000])
    assert sum(ix.local.size() for ix in ranks) == len(base)
    qd = torch.from_numpy(q).cuda()
    # the probe split across the ranks, then exchanged, as search_device does
    probes = ShardedIvfPqIndex.probe_table(torch.stack([ix.probe_slice(qd) for ix in ranks]), qd.shape[0])
    assert torch.equal(probes, single.probe_device(qd))
    gathered = torch.stack([ix.approx_candidates(qd, k, probes) for ix in ranks])
    assert torch.equal(gathered, torch.stack([ix.approx_candidates(qd, k) for ix in ranks]))
    mine = torch.stack([ix.rerank_owned(qd, k, gathered) for ix in ranks])
    d, r = ShardedIvfPqIndex.merge_final(mine, k)
    torch.cuda.synchronize()
    assert np.array_equal(r.cpu().numpy(), r_ref) and np.array_equal(d.cpu().numpy(), d_ref)
    # Bounds shared by the ranks' scans (one after another here, so later
    # ranks start from the earlier ones' tight bounds): the merged R best and
    # the final result are unchanged.
    from elips_b200.exact import merge_candidates_device
    bound = torch.full((qd.shape[0],), -1, dtype=torch.int32, device="cuda")
    shared = torch.stack([ix.approx_candidates(qd, k, probes, shared_bound=bound.data_ptr()) for ix in ranks])
    rk = 4 * k
    ua, ub = merge_candidates_device(gathered, world, rk, "dot_product")
    sa, sb = merge_candidates_device(shared, world, rk, "dot_product")
    assert torch.equal(ub, sb) and torch.equal(ua.view(torch.int32), sa.view(torch.int32))
    assert int((bound != -1).sum()) == qd.shape[0]        # every query's bound was tightened
    mine = torch.stack([ix.rerank_owned(qd, k, shared) for ix in ranks])
    d, r = ShardedIvfPqIndex.merge_final(mine, k)
    torch.cuda.synchronize()
    assert np.array_equal(r.cpu().numpy(), r_ref) and np.array_equal(d.cpu().numpy(), d_ref)


@pytest.mark.parametrize("flat", [False, True])
def test_replicated_query_slices_equal_whole_batch(model, flat):
    """Replicate mode (DistributedMode::replicate) over an IVF index: each
    replica answers a query_range slice of the batch (ranks emulated on one
    GPU); every query's ids and distances equal the whole batch's, the
    tie-heavy model included."""
    import torch
    from elips_b200.distributed import query_range
    from elips_b200.ivfpq import IvfFlatIndex, IvfPqIndex
    m = model
    ix = (IvfFlatIndex("euclidean", 64, m["cent"], nprobe=8) if flat
          else IvfPqIndex("euclidean", 64, m["cent"], m["cb"], nprobe=8))
    ix.add(m["base"], m["asg"])
    qd = torch.from_numpy(m["queries"]).cuda()
    d_ref, r_ref = ix.search_device(qd, 10)
    for world in (2, 3, 8):
        parts = [ix.search_device(qd[lo:hi], 10) for lo, hi in (query_range(qd.shape[0], r, world)
                                                                 for r in range(world))]
        torch.cuda.synchronize()
        assert torch.equal(torch.cat([p[1] for p in parts]), r_ref)
        assert torch.equal(torch.cat([p[0] for p in parts]).view(torch.int32), d_ref.view(torch.int32))
