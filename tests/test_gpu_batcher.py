"""DynamicBatcher on the device exact index (through the C ABI): concurrent
single-query callers, coalesced into batched launches, get exactly the
results of a direct batch search (src/gpu_engine/DynamicBatcher.cpp:67-106
hands each caller its row of the batch result)."""
import threading

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run_threads(batcher, queries, ks, threads):
    out = [None] * len(queries)
    errs = []

    def work(t):
        try:
            for i in range(t, len(queries), threads):
                out[i] = batcher.search(queries[i], ks[i])
        except Exception as e:  # surfaced below
            errs.append(e)

    ts = [threading.Thread(target=work, args=(t,)) for t in range(threads)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errs, errs
    return out


@pytest.mark.parametrize("precision,metric", [("int8", "dot_product"), ("fp16", "cosine"), ("fp32", "euclidean")])
def test_batched_equals_direct(precision, metric):
    from elips_b200 import DynamicBatcher, ExactIndex
    rng = np.random.default_rng(1)
    if precision == "int8":
        base = rng.integers(-127, 128, size=(20000, 128), dtype=np.int8)
        q = rng.integers(-127, 128, size=(300, 128), dtype=np.int8)
    else:
        base = rng.standard_normal((20000, 128)).astype(np.float32)
        q = rng.standard_normal((300, 128)).astype(np.float32)
    ix = ExactIndex(metric, 128, precision=precision)
    ix.add(base)
    d_ref, r_ref = ix.search_batch(q, 40)
    ks = [int(k) for k in rng.integers(1, 41, size=len(q))]
    b = DynamicBatcher(ix, window_us=2000, max_batch=64)
    res = _run_threads(b, q, ks, threads=24)
    for i, (d, r) in enumerate(res):
        k = ks[i]
        assert np.array_equal(r, r_ref[i, :k]) and np.array_equal(d, d_ref[i, :k]), i
    st = b.stats()
    assert st["queries_coalesced"] == len(q)
    assert st["kernel_launches"] < len(q), st  # concurrent callers were coalesced
    b.close()


def test_batcher_sequential_caller_and_dimension_check():
    from elips_b200 import DimensionMismatch, DynamicBatcher, ExactIndex
    rng = np.random.default_rng(2)
    base = rng.integers(-127, 128, size=(1000, 64), dtype=np.int8)
    ix = ExactIndex("dot_product", 64, precision="int8")
    ix.add(base)
    b = DynamicBatcher(ix, window_us=0, max_batch=8)
    d_ref, r_ref = ix.search_batch(base[:5], 3)
    for i in range(5):
        d, r = b.search(base[i], 3)
        assert np.array_equal(r, r_ref[i]) and np.array_equal(d, d_ref[i])
    with pytest.raises(DimensionMismatch):
        b.search(base[0, :10], 3)
    assert b.stats()["kernel_launches"] == 5
    b.close()


def test_flush_serves_pending_without_the_window():
    """DynamicBatcher::flush (DynamicBatcher.cpp:36-65): with a 20 s window
    and a batch limit far above the callers, queries wait for the window
    until flush() dispatches them; flush returns once they are served, and
    flush on an idle batcher returns at once."""
    import time
    from elips_b200 import DynamicBatcher, ExactIndex
    rng = np.random.default_rng(3)
    base = rng.standard_normal((5000, 64)).astype(np.float32)
    q = rng.standard_normal((6, 64)).astype(np.float32)
    ix = ExactIndex("euclidean", 64, precision="fp32")
    ix.add(base)
    d_ref, r_ref = ix.search_batch(q, 10)
    b = DynamicBatcher(ix, window_us=20_000_000, max_batch=1000)
    t0 = time.perf_counter()
    b.flush()
    assert time.perf_counter() - t0 < 1.0
    out = [None] * len(q)

    def work(i):
        out[i] = b.search(q[i], 10)

    ts = [threading.Thread(target=work, args=(i,)) for i in range(len(q))]
    for t in ts:
        t.start()
    deadline = time.perf_counter() + 10.0
    while b.pending() < len(q) and time.perf_counter() < deadline:
        time.sleep(0.01)
    assert b.pending() == len(q)                # every caller is queued
    assert all(o is None for o in out)          # still inside the window
    t0 = time.perf_counter()
    b.flush()
    assert time.perf_counter() - t0 < 5.0
    for t in ts:
        t.join(timeout=5.0)
    assert all(o is not None for o in out)
    for i, (d, r) in enumerate(out):
        assert np.array_equal(r, r_ref[i]) and np.array_equal(d, d_ref[i])
    b.close()
