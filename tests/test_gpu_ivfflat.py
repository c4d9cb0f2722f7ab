"""IVF-Flat parity (through the C ABI) with the reference's GpuIVFFlatIndex
(src/gpu_engine/GpuIVFFlatIndex.cpp:44-164), run here from its own compiled
sources (oracle/_ref): ids and distances identical on every query, ties
included (both order them by gather position)."""
import numpy as np
import pytest

import oracle as O
from tests import helpers as H

pytestmark = pytest.mark.gpu


def _same(d, r, d_ref, r_ref):
    """Rows identical; distances identical where a row exists (padding is +inf
    on the device, 0 in the reference's driver)."""
    return np.array_equal(r, r_ref) and np.array_equal(np.where(r >= 0, d, 0), np.where(r_ref >= 0, d_ref, 0))


@pytest.fixture(scope="module")
def model():
    return H.ivfpq_tie_model()


@pytest.mark.parametrize("metric", ["euclidean", "cosine", "dot_product"])
@pytest.mark.parametrize("nprobe,k", [(8, 10), (1, 5), (200, 3), (16, 100)])
def test_ivfflat_matches_reference(model, metric, nprobe, k, nthreads):
    from elips_b200.ivfpq import IvfFlatIndex
    base, q = model["base"], model["queries"]
    if metric != "euclidean":
        base, q = H.normalize(base), H.normalize(q)
    cent = model["cent"]
    asg = O.ivf_assign(metric, base, cent)
    ix = IvfFlatIndex(metric, 64, cent, nprobe=nprobe)
    ix.add(base[:30000], asg[:30000])
    ix.add(base[30000:], asg[30000:])
    d, r = ix.search_batch(q, k)
    d_ref, r_ref = O.RefIvfFlatIndex(metric, cent, asg, base, nprobe).search(q, k, nthreads)
    bad = [i for i in range(len(q)) if not _same(d[i], r[i], d_ref[i], r_ref[i])]
    assert not bad, f"{len(bad)} queries differ, first {bad[:5]}"


def test_ivfflat_single_query_and_fewer_candidates_than_k(model):
    from elips_b200.ivfpq import IvfFlatIndex
    base, cent = model["base"][:2000], model["cent"]
    asg = O.ivf_assign("euclidean", base, cent)
    ix = IvfFlatIndex("euclidean", 64, cent, nprobe=1)
    ix.add(base, asg)
    q = model["queries"][:1]
    d, r = ix.search_batch(q, 1000)
    d_ref, r_ref = O.ivfflat_search("euclidean", cent, base, asg, q, 1, 1000)
    assert _same(d[0], r[0], d_ref[0], r_ref[0])
    assert (r[0] == -1).any()


def test_ivfflat_device_api_odd_dimension():
    import torch
    from elips_b200.ivfpq import IvfFlatIndex
    d = 37
    cent = H.gaussian(20, d, seed=81)
    base = H.mixture(5000, d, cent, 0.3, seed=82)
    q = H.mixture(33, d, cent, 0.3, seed=83)
    asg = O.ivf_assign("euclidean", base, cent)
    ix = IvfFlatIndex("euclidean", d, cent, nprobe=3)
    ix.add_device(torch.from_numpy(base).cuda(), torch.from_numpy(asg.view(np.int32)).cuda())
    dist, rows = ix.search_device(torch.from_numpy(q).cuda(), 9)
    torch.cuda.synchronize()
    d_ref, r_ref = O.ivfflat_search("euclidean", cent, base, asg, q, 3, 9)
    assert _same(dist.cpu().numpy(), rows.cpu().numpy(), d_ref, r_ref)


def test_ivfflat_empty_index(model):
    from elips_b200.ivfpq import IvfFlatIndex
    ix = IvfFlatIndex("euclidean", 64, model["cent"], nprobe=4)
    d, r = ix.search_batch(model["queries"][:3], 5)
    assert (r == -1).all()
