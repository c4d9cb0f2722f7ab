"""The no-allocation exact search entry point, called through the C ABI.

elips_b200_exact_search_noalloc serves callers that cannot allocate device
memory at search time (a device already fully reserved by another allocator,
or a latency-critical path where an allocation may synchronise the device).
It draws its scratch from one fixed 64 MiB device array instead. These tests
check, on two calls in a row (the array keeps the previous call's contents),
that it returns what the allocating entry point returns, and that a call
needing more than the fixed array is refused with a clear status.

This file is collected last on purpose, so that a run stopping at the first
failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest

from tests import helpers as H

pytestmark = pytest.mark.gpu


def _noalloc(ix, q, k, mask=None):
    import torch
    from elips_b200 import _capi
    nq = q.shape[0]
    d = torch.empty((nq, k), dtype=torch.float32, device=q.device)
    r = torch.empty((nq, k), dtype=torch.int64, device=q.device)
    s = torch.cuda.current_stream(q.device).cuda_stream
    status = _capi.LIB.elips_b200_exact_search_noalloc(
        ix._h, q.data_ptr(), nq, k, mask.data_ptr() if mask is not None else None,
        d.data_ptr(), r.data_ptr(), s)
    return status, d, r


@pytest.mark.parametrize("metric,precision,n,dim,nq,k", [
    ("euclidean", "fp32", 40_000, 64, 300, 25),
    ("cosine", "fp16", 60_000, 768, 130, 100),
    ("euclidean", "bf16", 50_000, 384, 64, 20),
])
def test_noalloc_matches_allocating_search_two_calls(metric, precision, n, dim, nq, k):
    import torch
    from elips_b200 import ExactIndex, _capi
    base = H.gaussian(n, dim, seed=31)
    queries = H.gaussian(nq, dim, seed=32)
    if metric == "cosine":
        base, queries = H.normalize(base), H.normalize(queries)
    ix = ExactIndex(metric, dim, precision=precision)
    ix.add(base)
    qd = torch.from_numpy(queries).cuda()
    mask = None
    if precision == "bf16":
        words, _ = H.bernoulli_mask(n, 0.1, seed=33)
        mask = torch.from_numpy(words.view(np.int32)).cuda()
    d_ref, r_ref = ix.search_device(qd, k, mask=mask)
    torch.cuda.synchronize()
    d_ref, r_ref = d_ref.cpu().numpy(), r_ref.cpu().numpy()
    for _ in range(2):
        status, d, r = _noalloc(ix, qd, k, mask)
        assert status == _capi.OK, _capi.status_name(status)
        torch.cuda.synchronize()
        d, r = d.cpu().numpy(), r.cpu().numpy()
        # same slots; distances within the fp32 tolerance the parity tests use
        assert np.array_equal(r, r_ref)
        np.testing.assert_allclose(d, d_ref, rtol=1e-5, atol=1e-6)
    assert _capi.device_error(0) == 0


def test_noalloc_rejects_batches_beyond_its_fixed_scratch():
    import torch
    from elips_b200 import ExactIndex, _capi
    ix = ExactIndex("euclidean", 512, precision="fp32")
    ix.add(H.gaussian(1000, 512, seed=34))
    # 40,000 fp32 queries x 512 dims need 160 MiB of operand scratch alone
    qd = torch.zeros((40_000, 512), dtype=torch.float32, device="cuda")
    status, _, _ = _noalloc(ix, qd, 10)
    assert status == _capi.INVALID_ARGUMENT
    # the entry point still works afterwards
    q_small = torch.from_numpy(H.gaussian(8, 512, seed=35)).cuda()
    status, d, r = _noalloc(ix, q_small, 10)
    assert status == _capi.OK
    torch.cuda.synchronize()
    d_ref, r_ref = ix.search_batch(q_small.cpu().numpy(), 10)
    assert np.array_equal(r.cpu().numpy(), r_ref)
