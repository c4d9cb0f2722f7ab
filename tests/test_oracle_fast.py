"""The blocked exact-search oracle (oracle/oracle_fast.c) returns exactly what
the scalar restatement (oracle/oracle.c, itself pinned to the reference's
ExactIndex::search) returns: same rows, same distance bits, ties included.
The large-shape parity checks rely on it."""
import numpy as np
import pytest

import oracle as O


def _base(rng, n, d, metric):
    b = rng.standard_normal((n, d)).astype(np.float32)
    t = min(40, n // 2)
    b[n // 2:n // 2 + t] = b[:t]                        # exact ties
    if metric == "cosine":
        b /= np.linalg.norm(b, axis=1, keepdims=True)
    return b


@pytest.mark.parametrize("metric", ["cosine", "euclidean", "dot_product"])
@pytest.mark.parametrize("n,d,nq,k", [(3001, 77, 37, 10), (9000, 128, 70, 100), (1500, 768, 17, 5),
                                      (40, 16, 3, 64)])
@pytest.mark.parametrize("masked", [False, True])
def test_fast_exact_equals_scalar(metric, n, d, nq, k, masked):
    rng = np.random.default_rng(n + d + nq)
    b = _base(rng, n, d, metric)
    q = rng.standard_normal((nq, d)).astype(np.float32)
    q[0] = b[3]
    mask = rng.integers(0, 2 ** 32, (n + 31) // 32, dtype=np.uint64).astype(np.uint32) if masked else None
    d1, r1 = O.exact_search(metric, b, q, k, mask=mask)
    d2, r2 = O.exact_search_fast(metric, b, q, k, mask=mask)
    assert np.array_equal(r1, r2)
    assert np.array_equal(d1.view(np.uint32), d2.view(np.uint32))


@pytest.mark.parametrize("n,d,nq,k", [(5000, 64, 33, 10), (4000, 1024, 20, 50), (3001, 100, 17, 5),
                                      (30, 40, 2, 64)])
def test_fast_int8_equals_scalar(n, d, nq, k):
    rng = np.random.default_rng(n + d)
    b = rng.integers(-127, 128, (n, d), dtype=np.int8)
    t = min(20, n // 2)
    b[n // 2:n // 2 + t] = b[:t]
    q = rng.integers(-127, 128, (nq, d), dtype=np.int8)
    d1, r1 = O.int8_ip_search(b, q, k)
    d2, r2 = O.int8_ip_search_fast(b, q, k)
    assert np.array_equal(r1, r2)
    assert np.array_equal(d1.view(np.uint32), d2.view(np.uint32))
