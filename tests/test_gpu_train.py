"""Index build on the device (through the C ABI) against the oracle's
restatements of the reference's trainers, bit for bit:

* quant::detail::kmeans / train_pq_codebook (src/quant_engine/KMeans.cpp:182-268)
* IvfIndexState::train_centroids + assign_vectors_to_centroids
  (src/gpu_engine/detail/IvfIndexState.cpp:118-208)
* GpuIVFPQIndex's model build (GpuIVFPQIndex.cpp:88-131)

The restatements are themselves pinned to the reference's own compiled code
(tests/test_oracle_pin.py); here the larger cases also cover empty lists,
duplicate rows (equal distances) and subspaces that stop early."""
import numpy as np
import pytest

import oracle as O
from tests import helpers as H

pytestmark = pytest.mark.gpu

METRICS = ["euclidean", "cosine", "dot_product"]


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _rows(n, d, seed, metric="euclidean", clusters=48, sigma=0.3):
    cents = H.gaussian(clusters, d, seed=seed)
    x = H.mixture(n, d, cents, sigma, seed=seed + 1)
    return H.normalize(x) if metric == "cosine" else x


@pytest.mark.parametrize("n,d,k,iters", [(20000, 16, 64, 10), (5000, 37, 100, 6), (300, 8, 256, 4)])
def test_kmeans_bit_exact(n, d, k, iters):
    from elips_b200 import train
    x = _rows(n, d, seed=11)
    assert np.array_equal(_bits(train.kmeans(x, k, iters)), _bits(O.kmeans(x, k, iters)))


def test_kmeans_duplicates_and_empty_clusters():
    """Few distinct rows: many seeds coincide, ties everywhere, clusters go
    empty and are reseeded from row c % n."""
    from elips_b200 import train
    rng = np.random.default_rng(5)
    distinct = rng.standard_normal((7, 12)).astype(np.float32)
    x = distinct[rng.integers(0, 7, 3000)]
    for k, iters in [(32, 5), (7, 3), (64, 0)]:
        assert np.array_equal(_bits(train.kmeans(x, k, iters)), _bits(O.kmeans(x, k, iters)))


@pytest.mark.parametrize("n,d,m,ksub", [(8000, 32, 4, 256), (3000, 24, 3, 16), (200, 16, 8, 256)])
def test_train_pq_codebook_bit_exact(n, d, m, ksub):
    from elips_b200 import train
    x = _rows(n, d, seed=21)
    got = train.train_pq_codebook(x, m, ksub, 10)
    assert np.array_equal(_bits(got), _bits(O.train_pq_codebook(x, m, ksub, 10)))


@pytest.mark.parametrize("metric", METRICS)
def test_ivf_assign_bit_exact(metric):
    from elips_b200 import train
    x = _rows(30000, 40, seed=31, metric=metric)
    cent = _rows(300, 40, seed=32, metric=metric)
    cent[17] = cent[250]          # duplicate list: the lower index must win
    cent[90] = cent[3]
    assert np.array_equal(train.ivf_assign(metric, x, cent), O.ivf_assign(metric, x, cent))


@pytest.mark.parametrize("metric", METRICS)
@pytest.mark.parametrize("n,d,nlist,iters", [(20000, 32, 64, 5), (4000, 20, 500, 3), (1000, 8, 1000, 1)])
def test_ivf_train_bit_exact(metric, n, d, nlist, iters):
    from elips_b200 import train
    x = _rows(n, d, seed=41, metric=metric)
    c, a = train.ivf_train(metric, x, nlist, iters)
    c_ref, a_ref = O.ivf_train(metric, x, nlist, iters)
    assert np.array_equal(_bits(c), _bits(c_ref)) and np.array_equal(a, a_ref)


def test_ivf_train_requested_lists_above_rows():
    """rebuild_from_current_data trains max(1, min(requested, n)) lists."""
    from elips_b200 import train
    x = _rows(50, 8, seed=51)
    c, a = train.ivf_train("euclidean", x, 4096, 2)
    c_ref, a_ref = O.ivf_train("euclidean", x, 50, 2)
    assert c.shape == (50, 8) and np.array_equal(_bits(c), _bits(c_ref)) and np.array_equal(a, a_ref)


@pytest.mark.parametrize("metric", ["euclidean", "cosine"])
def test_ivfpq_train_matches_composition(metric):
    """ivf_train, residuals, train_pq_codebook(10), encode_pq: each stage of
    the oracle in sequence gives the device build's outputs bit for bit."""
    from elips_b200 import train
    x = _rows(12000, 32, seed=61, metric=metric)
    c, a, cb, codes = train.ivfpq_train(metric, x, 40, 4, pq_dim=8, pq_bits=8)
    c_ref, a_ref = O.ivf_train(metric, x, 40, 4)
    assert np.array_equal(_bits(c), _bits(c_ref)) and np.array_equal(a, a_ref)
    res = (x - c_ref[a_ref]).astype(np.float32)
    cb_ref = O.train_pq_codebook(res, 8, 256, 10)
    assert np.array_equal(_bits(cb), _bits(cb_ref))
    assert np.array_equal(codes, O.encode_pq(cb_ref, res))


def test_ivf_train_device_tensors_large():
    """A 400k x 64 build with 512 lists through the device entry point: every
    sampled row's list is its nearest centroid by the oracle's distance, and
    the final assignment equals a fresh assignment against the centroids."""
    import torch
    from elips_b200 import train
    x = _rows(400_000, 64, seed=71, clusters=600)
    xt = torch.from_numpy(x).cuda()
    c, a = train.ivf_train_device("euclidean", xt, 512, 3)
    torch.cuda.synchronize()
    c, a = c.cpu().numpy(), a.cpu().numpy().astype(np.uint32)
    rng = np.random.default_rng(3)
    pick = rng.choice(len(x), 3000, replace=False)
    assert np.array_equal(a[pick], O.ivf_assign("euclidean", x[pick], c))
    assert np.array_equal(train.ivf_assign("euclidean", x, c), a)


@pytest.mark.parametrize("metric", METRICS)
def test_ivf_nearest_distances_bit_exact(metric):
    """The argmin kernel's winning distance for every row equals
    elips::distance(row, its centroid) bit for bit: every sequential chain is
    rounded as the reference's scalar loop (a fused multiply-add anywhere would
    show up here even where it does not change the argmin)."""
    from elips_b200 import train
    x = _rows(4000, 72, seed=81, metric=metric)
    cent = _rows(130, 72, seed=82, metric=metric)
    a, dist = train.ivf_nearest(metric, x, cent)
    assert np.array_equal(a, O.ivf_assign(metric, x, cent))
    ref = np.array([O.distance(metric, x[i], cent[a[i]]) for i in range(len(x))], np.float32)
    assert np.array_equal(_bits(dist), _bits(ref))
