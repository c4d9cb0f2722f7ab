"""The GpuPort boundary as ELIPS would use it: the reference's own index
classes (GpuBruteForceIndex, GpuIVFFlatIndex, GpuIVFPQIndex; compiled from its
sources into oracle/_ref/libelips_ref_b200.so) run on
elips::gpu::cuda::CudaBackend (elips_b200/integration/CudaBackend.cpp, the
adapter over this library's C ABI) and on the CPU GpuPort. Every
compute_distances_batch / top_k the reference issues then goes through the
B200 library; results must be identical, ids and distances, on every query.
Searches run on 4 threads at once, as Vault::seek's readers call an index."""
import numpy as np
import pytest

import oracle as O
from tests import helpers as H

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not O.REF_B200_SO.exists(), reason="reference-on-B200 driver not built")]


@pytest.fixture(scope="module")
def model():
    return H.ivfpq_tie_model()


@pytest.mark.parametrize("metric", ["euclidean", "cosine", "dot_product"])
def test_brute_force_index_on_the_b200_port(metric):
    base = H.gaussian(4000, 48, seed=91)
    q = H.gaussian(40, 48, seed=92)
    if metric == "cosine":
        base, q = H.normalize(base), H.normalize(q)
    cpu = O.RefBruteForceIndex(metric, base, port="cpu")
    b200 = O.RefBruteForceIndex(metric, base, port="b200")
    for k in (1, 10, 4000):
        d1, r1 = cpu.search(q, k, 4)
        d2, r2 = b200.search(q, k, 4)
        assert np.array_equal(r1, r2) and np.array_equal(d1, d2)
        d3, r3 = cpu.search_batch(q, k)
        d4, r4 = b200.search_batch(q, k)
        assert np.array_equal(r3, r4) and np.array_equal(d3, d4)


def test_ivf_flat_index_on_the_b200_port(model):
    m = model
    asg = O.ivf_assign("euclidean", m["base"], m["cent"])
    cpu = O.RefIvfFlatIndex("euclidean", m["cent"], asg, m["base"], 8, port="cpu")
    b200 = O.RefIvfFlatIndex("euclidean", m["cent"], asg, m["base"], 8, port="b200")
    q = m["queries"][:80]
    d1, r1 = cpu.search(q, 10, 4)
    d2, r2 = b200.search(q, 10, 4)
    assert np.array_equal(r1, r2) and np.array_equal(d1, d2)
    d3, r3 = b200.search_batch(q, 10)
    assert np.array_equal(r1, r3) and np.array_equal(d1, d3)


def test_ivf_pq_index_on_the_b200_port(model):
    m = model
    args = ("euclidean", m["cent"], m["asg"], m["cb"], m["codes"], m["base"], 8)
    cpu = O.RefIvfPqIndex(*args, port="cpu")
    b200 = O.RefIvfPqIndex(*args, port="b200")
    q = m["queries"][:80]
    d1, r1 = cpu.search(q, 10, 4)
    d2, r2 = b200.search(q, 10, 4)
    assert np.array_equal(r1, r2) and np.array_equal(d1, d2)


@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 0), (0, 1), (1, 1)])
def test_gemm_fp32_matches_float64(ta, tb):
    """CudaBackend::gemm_fp32 runs on the library's fp32 kernel: row-major
    C = op(A) op(B) within fp32 rounding of a float64 product."""
    from elips_b200 import _capi
    rng = np.random.default_rng(7 + 2 * ta + tb)
    m, n, kk = 70, 131, 45
    a = rng.standard_normal((kk, m) if ta else (m, kk)).astype(np.float32)
    b = rng.standard_normal((n, kk) if tb else (kk, n)).astype(np.float32)
    c = np.empty((m, n), np.float32)
    assert _capi.LIB.elips_b200_gemm_fp32(0, a.ctypes.data, b.ctypes.data, c.ctypes.data, m, n, kk, ta, tb, 0,
                                          None) == 0
    ref = (a.T if ta else a).astype(np.float64) @ (b.T if tb else b).astype(np.float64)
    np.testing.assert_allclose(c, ref, rtol=1e-5, atol=1e-4)
