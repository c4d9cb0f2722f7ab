"""Bounded device waits (every mbarrier wait in the kernels has a cycle
budget): a wait whose barrier nothing completes expires, records the device
error word, and the host reports ELIPS_B200_DEVICE_TIMEOUT; the context stays
usable and the next search is correct. The expiry is made with a short
budget on a barrier nothing arrives on (elips_b200_wait_selftest), the same
wait routine the pipelines use; no fault, no trap, no unbounded spin."""
import numpy as np
import pytest

import oracle as O
from tests import helpers as H

pytestmark = pytest.mark.gpu


def test_wait_expires_reports_timeout_and_context_stays_usable():
    from elips_b200 import ExactIndex, _capi
    # ~0.5 ms at the B200's clock: the wait must give up and say so
    assert _capi.LIB.elips_b200_wait_selftest(0, 1_000_000) == _capi.DEVICE_TIMEOUT
    assert _capi.device_error(0) == 0                  # the error word was read and cleared
    assert _capi.LIB.elips_b200_wait_selftest(0, 1) == _capi.DEVICE_TIMEOUT
    assert _capi.LIB.elips_b200_wait_selftest(0, 0) == _capi.INVALID_ARGUMENT
    assert _capi.LIB.elips_b200_wait_selftest(0, 1 << 40) == _capi.INVALID_ARGUMENT
    # the next search runs normally and matches the oracle
    base = H.gaussian(5000, 64, seed=401)
    q = H.gaussian(300, 64, seed=402)
    ix = ExactIndex("euclidean", 64, precision="fp32")
    ix.add(base)
    d, r = ix.search_batch(q, 10)
    rd, rr = O.exact_search("euclidean", base, q, 10)
    H.assert_ranked_match(d, r, rd, rr, lambda qi, row: O.distance("euclidean", q[qi], base[row]), rtol=1e-5)
    assert _capi.device_error(0) == 0
