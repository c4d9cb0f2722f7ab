"""The C restatement (oracle/oracle.c) against golden outputs of the
reference's own compiled code (tests/golden/reference_outputs.npz, made by
tests/golden/make_golden.py), and the known answers of the reference's unit
tests. Runs on CPU without the reference sources."""
from pathlib import Path

import numpy as np
import pytest

import oracle as O

G = np.load(Path(__file__).resolve().parent / "golden" / "reference_outputs.npz")
METRICS = ["cosine", "euclidean", "dot_product"]


@pytest.mark.parametrize("metric", METRICS)
def test_exact_golden(metric):
    b, q = (G["unit_base"], G["unit_queries"]) if metric == "cosine" else (G["base"], G["queries"])
    d, r = O.exact_search(metric, b, q, 7, nthreads=1)
    assert np.array_equal(d, G[f"exact_{metric}_dist"])
    assert np.array_equal(r, G[f"exact_{metric}_rows"])


def test_sq8_codes_golden():
    assert np.array_equal(O.sq8_encode(G["sq8_mins"], G["sq8_scales"], G["base"]), G["sq8_codes"])
    m, s = O.sq8_train(G["base"][:300])
    assert np.array_equal(m, G["sq8_mins"]) and np.array_equal(s, G["sq8_scales"])


@pytest.mark.parametrize("metric", METRICS)
def test_sq8_golden(metric):
    d, r = O.sq8_search(metric, G["sq8_mins"], G["sq8_scales"], G["sq8_codes"], G["queries"], 5, nthreads=1)
    assert np.array_equal(d, G[f"sq8_{metric}_dist"]) and np.array_equal(r, G[f"sq8_{metric}_rows"])


@pytest.mark.parametrize("metric", METRICS)
def test_pq_golden(metric):
    assert np.array_equal(O.encode_pq(G["pq_codebook"], G["base"]), G["pq_codes"])
    d, r = O.pq_search(metric, G["pq_codebook"], G["pq_codes"], G["queries"], 5, nthreads=1)
    assert np.array_equal(d, G[f"pq_{metric}_dist"]) and np.array_equal(r, G[f"pq_{metric}_rows"])


@pytest.mark.parametrize("metric", METRICS)
def test_opq_golden(metric):
    rot = G["opq_rotation"]
    codes = O.encode_pq(G["pq_codebook"], O.rotate_rows(rot, G["base"]))
    d, r = O.pq_search(metric, G["pq_codebook"], codes, O.rotate_rows(rot, G["queries"]), 5, nthreads=1)
    assert np.array_equal(d, G[f"opq_{metric}_dist"]) and np.array_equal(r, G[f"opq_{metric}_rows"])


def test_kmeans_golden():
    assert np.array_equal(O.kmeans(G["base"], 10, 8), G["kmeans_centroids"])


def test_ivfpq_golden():
    assert np.array_equal(O.ivf_assign("euclidean", G["base"], G["ivf_centroids"]), G["ivf_assignments"])
    d, r = O.ivfpq_search("euclidean", G["ivf_centroids"], G["ivf_codebook"], G["ivf_codes"], G["base"],
                          G["ivf_assignments"], G["queries"], 3, 4, nthreads=1)
    assert np.array_equal(d, G["ivf_dist"]) and np.array_equal(r, G["ivf_rows"])


# Known answers from the reference's unit tests (tests/unit/metrics_test.cpp:13-40,
# tests/unit/exact_edge_cases_test.cpp:20-97, tests/unit/gpu/GpuAdvancedIndexTest.cpp:20-31).

def test_metrics_known_answers():
    assert abs(O.distance("cosine", [1, 0], [1, 0])) < 1e-6
    assert abs(O.distance("cosine", [1, 0], [0, 1]) - 1.0) < 1e-6
    assert abs(O.distance("euclidean", [0, 0], [3, 4]) - 5.0) < 1e-6
    assert abs(O.distance("dot_product", [1, 2, 3], [1, 1, 1]) + 6.0) < 1e-6


def test_exact_edge_known_answers():
    d, r = O.exact_search("euclidean", np.zeros((0, 3), np.float32), np.array([[1, 0, 0]], np.float32), 10)
    assert (r == -1).all()
    base = np.array([[0, 0], [1, 0], [2, 0]], np.float32)
    d, r = O.exact_search("euclidean", base, np.array([[0, 0]], np.float32), 100)
    assert list(r[0, :3]) == [0, 1, 2] and (r[0, 3:] == -1).all()
    for m in METRICS:
        d, r = O.exact_search(m, np.array([[1, 0]], np.float32), np.array([[1, 0]], np.float32), 1)
        assert r[0, 0] == 0


def test_gpu_advanced_sample_known_answers():
    sample = np.array([[0, 0, 0, 0], [0.1, 0.1, 0, 0], [5, 5, 5, 5], [5.2, 5.1, 5, 5],
                       [-4, -4, -4, -4], [-4.1, -4, -4, -4]], np.float32)
    q = np.array([[0, 0, 0, 0], [5.2, 5.1, 5, 5], [-4.1, -4, -4, -4], [0.1, 0.1, 0, 0]], np.float32)
    d, r = O.exact_search("euclidean", sample, q, 2)
    assert [int(x) for x in r[:, 0]] == [0, 3, 5, 1]
