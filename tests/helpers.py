"""Seeded synthetic data with the shapes and distributions of the benchmark
configurations, and the parity comparators the tests share."""
from __future__ import annotations

import numpy as np


def gaussian(n, d, seed):
    return np.random.default_rng(seed).standard_normal((n, d), dtype=np.float32)


def normalize(x):
    """Vector::normalized (include/elips/domain/Vector.hpp:34-44): x / |x| in fp32."""
    x = np.asarray(x, np.float32)
    mag = np.sqrt(np.einsum("ij,ij->i", x, x, dtype=np.float32)).astype(np.float32)
    mag[mag == 0] = 1.0
    return (x / mag[:, None]).astype(np.float32)


def mixture(n, d, centroids, sigma, seed, normalized=False):
    """Gaussian mixture: centroid[u] + sigma * N(0, I), u uniform."""
    rng = np.random.default_rng(seed)
    c = centroids[rng.integers(0, centroids.shape[0], n)]
    x = (c + sigma * rng.standard_normal((n, d), dtype=np.float32)).astype(np.float32)
    return normalize(x) if normalized else x


def round_fp16(x):
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def round_bf16(x):
    x = np.ascontiguousarray(x, np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16   # round to nearest even
    return r.astype(np.uint32).view(np.float32).reshape(x.shape)


def bernoulli_mask(n, p, seed):
    bits = np.random.default_rng(seed).random(n) < p
    words = np.zeros((n + 31) // 32, np.uint32)
    idx = np.nonzero(bits)[0]
    np.bitwise_or.at(words, idx >> 5, (np.uint32(1) << (idx & 31).astype(np.uint32)))
    return words, bits


def recall(rows_gpu, rows_ref):
    hits = 0
    total = 0
    for a, b in zip(rows_gpu, rows_ref):
        b = b[b >= 0]
        total += len(b)
        hits += len(set(a[a >= 0].tolist()) & set(b.tolist()))
    return hits / max(total, 1)


def assert_ranked_match(dist_gpu, rows_gpu, dist_ref, rows_ref, true_dist, rtol, atol=0.0):
    """Same slots as the reference except where distances tie within rtol:
    at every rank the GPU's slot must have a true distance equal, within
    rtol, to the reference's distance at that rank, and the reported
    distances must agree within rtol."""
    valid_ref = rows_ref >= 0
    assert np.array_equal(rows_gpu >= 0, valid_ref), "different number of results"
    tol = rtol * np.maximum(np.abs(dist_ref), 1e-30) + atol
    bad = valid_ref & (np.abs(dist_gpu - dist_ref) > tol)
    assert not bad.any(), f"{bad.sum()} distances outside rtol={rtol}"
    diff = valid_ref & (rows_gpu != rows_ref)
    for q, i in zip(*np.nonzero(diff)):
        td = true_dist(q, int(rows_gpu[q, i]))
        assert abs(td - dist_ref[q, i]) <= tol[q, i], (
            f"query {q} rank {i}: slot {rows_gpu[q, i]} (true {td}) vs reference "
            f"slot {rows_ref[q, i]} ({dist_ref[q, i]})")
    for q in range(rows_gpu.shape[0]):
        r = rows_gpu[q][rows_gpu[q] >= 0]
        assert len(np.unique(r)) == len(r), f"duplicate slots for query {q}"


def ivfpq_tie_model():
    """IVF-PQ model whose lists hold many rows with identical residual codes
    (12.7k of 60k rows share a code with another row): coarse k-means leaves
    tight residual clusters, so approximate distances tie exactly at the
    rerank boundary for about a quarter of the queries. Trained with the
    reference's own k-means and PQ trainer (oracle/_ref)."""
    import oracle as O
    d, nlist = 64, 128
    cents = gaussian(nlist, d, seed=61)
    base = mixture(60_000, d, cents, 0.2, seed=62)
    queries = mixture(200, d, cents, 0.2, seed=63)
    cent = O.ref_kmeans(base[::10], nlist, 4)
    asg = O.ivf_assign("euclidean", base, cent)
    res = base - cent[asg]
    cb = O.ref_train_pq_codebook(res[::6], 8, 256, 4)
    codes = O.ref_encode_pq(cb, res)
    return dict(base=base, queries=queries, cent=cent, asg=asg, cb=cb, codes=codes)
