"""Pins the C restatement (oracle/oracle.c) to the reference's own compiled
code (oracle/_ref, built from the reference sources by oracle/Makefile):
bit-exact on seeded inputs, for every path the GPU kernels are checked on."""
import numpy as np
import pytest

import oracle as O
from tests import helpers as H

pytestmark = pytest.mark.skipif(not O.ref_available(), reason="reference sources not present")

METRICS = ["cosine", "euclidean", "dot_product"]


@pytest.fixture(scope="module")
def data():
    rng = np.random.default_rng(7)
    base = rng.standard_normal((3000, 48)).astype(np.float32)
    q = rng.standard_normal((40, 48)).astype(np.float32)
    return base, q


@pytest.mark.parametrize("metric", METRICS)
def test_distance_matches_reference(metric, data):
    base, q = data
    for i in range(20):
        assert O.distance(metric, q[i], base[i]) == O.ref_distance(metric, q[i], base[i])


@pytest.mark.parametrize("metric", METRICS)
def test_exact_search_matches_reference(metric, data):
    base, q = data
    d1, r1 = O.exact_search(metric, base, q, 17)
    d2, r2 = O.RefExactIndex(metric, base).search(q, 17)
    assert np.array_equal(d1, d2)
    assert np.array_equal(r1, r2)


def test_exact_search_k_above_n_pads(data):
    base, q = data
    d1, r1 = O.exact_search("euclidean", base[:5], q[:3], 9)
    d2, r2 = O.RefExactIndex("euclidean", base[:5]).search(q[:3], 9)
    assert np.array_equal(r1, r2)
    assert (r1[:, 5:] == -1).all()


def test_sq8_train_encode_match_reference(data):
    base, _ = data
    mins, scales = O.sq8_train(base)
    m2, s2 = O.ref_sq8_train("euclidean", base)
    assert np.array_equal(mins, m2) and np.array_equal(scales, s2)
    # out-of-range inserts clamp (ScalarQuantizer.cpp:61-66)
    probe = base * 1.5
    assert np.array_equal(O.sq8_encode(mins, scales, probe), O.ref_sq8_encode("euclidean", mins, scales, probe))


@pytest.mark.parametrize("metric", METRICS)
def test_sq8_search_matches_reference(metric, data):
    base, q = data
    mins, scales = O.sq8_train(base)
    codes = O.sq8_encode(mins, scales, base)
    d1, r1 = O.sq8_search(metric, mins, scales, codes, q, 10)
    d2, r2 = O.RefExactIndex(metric, base, codec="sq8", mins=mins, scales=scales).search(q, 10)
    assert np.array_equal(d1, d2) and np.array_equal(r1, r2)


@pytest.mark.parametrize("metric", METRICS)
def test_pq_search_matches_reference(metric, data):
    base, q = data
    cb = O.ref_train_pq_codebook(base, 8, 256, 4)
    codes = O.encode_pq(cb, base)
    assert np.array_equal(codes, O.ref_encode_pq(cb, base))
    d1, r1 = O.pq_search(metric, cb, codes, q, 10)
    d2, r2 = O.RefExactIndex(metric, base, codec="pq", codebook=cb, pq_bits=8).search(q, 10)
    assert np.array_equal(d1, d2) and np.array_equal(r1, r2)


def test_kmeans_matches_reference(data):
    base, _ = data
    assert np.array_equal(O.kmeans(base, 32, 6), O.ref_kmeans(base, 32, 6))


def test_ivfpq_search_matches_reference(data):
    base, q = data
    cent = O.ref_kmeans(base, 24, 6)
    asg = O.ivf_assign("euclidean", base, cent)
    res = base - cent[asg]
    cb = O.ref_train_pq_codebook(res, 8, 16, 10)
    codes = O.ref_encode_pq(cb, res)
    d1, r1 = O.ivfpq_search("euclidean", cent, cb, codes, base, asg, q, 5, 10)
    d2, r2 = O.RefIvfPqIndex("euclidean", cent, asg, cb, codes, base, 5, pq_bits=4).search(q, 10)
    assert np.array_equal(d1, d2) and np.array_equal(r1, r2)


@pytest.mark.parametrize("nprobe,k", [(8, 10), (1, 5), (200, 3)])
def test_ivfpq_tie_order_matches_reference(nprobe, k):
    """Candidates tied at the rerank boundary: the restatement of libstdc++'s
    partial_sort picks the same ones as the reference on every query, and
    the device order (ties by slot) differs from it only on tied queries."""
    m = H.ivfpq_tie_model()
    args = ("euclidean", m["cent"], m["cb"], m["codes"], m["base"], m["asg"], m["queries"], nprobe, k)
    d0, r0, gap = O.ivfpq_search(*args, order="reference", with_gap=True)
    d1, r1 = O.ivfpq_search(*args, order="device")
    d2, r2 = O.RefIvfPqIndex("euclidean", m["cent"], m["asg"], m["cb"], m["codes"], m["base"], nprobe).search(
        m["queries"], k)
    assert np.array_equal(d0, d2) and np.array_equal(r0, r2)
    assert (gap == 0).sum() >= 20  # the model really exercises boundary ties
    differ = [q for q in range(len(r1)) if not (np.array_equal(r1[q], r2[q]) and np.array_equal(d1[q], d2[q]))]
    assert all(gap[q] == 0 for q in differ)


@pytest.mark.parametrize("metric", METRICS)
def test_ivfflat_search_matches_reference(metric):
    """GpuIVFFlatIndex::search and search_batch, ties by gather position."""
    m = H.ivfpq_tie_model()
    base, q = m["base"][:20000], m["queries"][:60]
    if metric != "euclidean":
        base, q = H.normalize(base), H.normalize(q)
    asg = O.ivf_assign(metric, base, m["cent"])
    for nprobe, k in [(8, 10), (1, 5), (200, 3)]:
        d1, r1 = O.ivfflat_search(metric, m["cent"], base, asg, q, nprobe, k)
        ref = O.RefIvfFlatIndex(metric, m["cent"], asg, base, nprobe)
        d2, r2 = ref.search(q, k)
        d3, r3 = ref.search_batch(q, k)
        assert np.array_equal(d1, d2) and np.array_equal(r1, r2)
        assert np.array_equal(d2, d3) and np.array_equal(r2, r3)


def test_normalize_matches_reference():
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((300, 77)) * rng.uniform(1e-3, 1e3, (300, 1))).astype(np.float32)
    x[5] = 0.0
    x[6, :] = 0.0
    x[6, 3] = -0.0
    assert np.array_equal(O.normalize_rows(x).view(np.uint32), O.ref_normalize_rows(x).view(np.uint32))


@pytest.mark.parametrize("metric", METRICS)
def test_ivf_train_matches_reference(metric):
    """IvfIndexState::train_centroids + final assignment, restated vs the
    reference's own (GpuIVFFlatIndex::build_from_batch), bit-exact."""
    cents = H.gaussian(24, 16, seed=101)
    rows = H.mixture(3000, 16, cents, 0.3, seed=102)
    if metric == "cosine":
        rows = H.normalize(rows)
    c1, a1 = O.ivf_train(metric, rows, 24, 5)
    c2, a2 = O.ref_ivf_train(metric, rows, 24, 5)
    assert np.array_equal(c1.view(np.uint32), c2.view(np.uint32)) and np.array_equal(a1, a2)


def test_train_pq_codebook_matches_reference():
    rows = H.gaussian(4000, 24, seed=103)
    c1 = O.train_pq_codebook(rows, 3, 32, 10)
    c2 = O.ref_train_pq_codebook(rows, 3, 32, 10)
    assert np.array_equal(c1.view(np.uint32), c2.view(np.uint32))
