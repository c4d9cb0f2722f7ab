"""Row-sharded exact search with per-query admission bounds shared by the
shards (GpuDistributedIndex shard mode, src/gpu_engine/GpuDistributedIndex.cpp:
155-207): each shard's kernel reads and tightens one bound array while it
runs, so later shards admit only candidates that can still reach the global
top-k. The merged result must equal one index over all rows, ties by row.
Shards are emulated on one GPU here (searched one after the other, so later
shards start from the earlier ones' tight bounds); the 2-GPU test runs them
as processes that share the root's bounds over NVLink peer memory."""
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle as O
from tests import helpers as H

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("precision,metric,k", [("fp32", "euclidean", 10), ("fp16", "cosine", 100),
                                                ("int8", "dot_product", 50)])
def test_shared_bounds_merge_equals_single_index(precision, metric, k):
    import torch
    from elips_b200 import ExactIndex
    from elips_b200.distributed import shard_range
    from elips_b200.exact import merge_candidates_device
    n, d, nq, world = 60_000, 64, 300, 3
    if precision == "int8":
        rng = np.random.default_rng(71)
        base = rng.integers(-3, 4, (n, d), dtype=np.int8)          # many exact ties
        queries = rng.integers(-3, 4, (nq, d), dtype=np.int8)
    else:
        base = H.gaussian(n, d, seed=71)
        base[30_000:30_200] = base[:200]
        queries = H.gaussian(nq, d, seed=72)
        if metric == "cosine":
            base, queries = H.normalize(base), H.normalize(queries)
    whole = ExactIndex(metric, d, precision=precision)
    whole.add(base)
    d_ref, r_ref = whole.search_batch(queries, k)
    qd = torch.from_numpy(queries).cuda()
    bound = torch.full((nq,), -1, dtype=torch.int32, device="cuda")
    blocks = torch.empty((world, nq, k, 2), dtype=torch.int32, device="cuda")
    for r in range(world):
        lo, hi = shard_range(n, r, world)
        ix = ExactIndex(metric, d, precision=precision)
        ix.add(base[lo:hi])
        ix.search_candidates_shared_device(qd, k, lo, blocks[r], bound)
        torch.cuda.synchronize()
        ix.close()
    dist, rows = merge_candidates_device(blocks, world, k, metric)
    torch.cuda.synchronize()
    assert np.array_equal(rows.cpu().numpy(), r_ref)
    assert np.array_equal(dist.cpu().numpy().view(np.uint32), d_ref.view(np.uint32))


def _gpus():
    import torch
    return torch.cuda.device_count()


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_peer_exchange_two_processes_equals_single_index(tmp_path):
    """Two ranks (NCCL, one GPU each) search their row ranges with the bounds
    and candidate blocks in rank 0's memory; rank 0's merged result equals
    one index over all rows."""
    script = os.path.join(os.path.dirname(__file__), "peer_exchange_worker.py")
    out = tmp_path / "result.npz"
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT="29533", NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                        "--master-addr", "127.0.0.1", "--master-port", "29533", script, str(out)],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    got = np.load(out)
    from elips_b200 import ExactIndex
    base = H.gaussian(80_000, 96, seed=81)
    base[40_000:40_100] = base[:100]
    queries = H.gaussian(500, 96, seed=82)
    whole = ExactIndex("euclidean", 96, precision="fp32")
    whole.add(base)
    for k in (10, 100):
        d_ref, r_ref = whole.search_batch(queries, k)
        assert np.array_equal(got[f"rows{k}"], r_ref)
        assert np.array_equal(got[f"dist{k}"].view(np.uint32), d_ref.view(np.uint32))
    d_ref, r_ref = whole.search_batch(queries[:1], 20)
    assert np.array_equal(got["rows1"], r_ref)
    assert np.array_equal(got["dist1"].view(np.uint32), d_ref.view(np.uint32))


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_ivfpq_peer_exchange_two_processes_equals_single_index(tmp_path):
    """Two ranks (NCCL, one GPU each) of a list-sharded IVF-PQ index on the
    tie-heavy model: their scans share the per-query bounds in rank 0's
    memory and their k best reach rank 0 over peer memory; rank 0's result
    equals one index over all lists, ids and distances."""
    script = os.path.join(os.path.dirname(__file__), "ivfpq_peer_worker.py")
    out = tmp_path / "result.npz"
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT="29534", NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                        "--master-addr", "127.0.0.1", "--master-port", "29534", script, str(out)],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    got = np.load(out)
    from elips_b200.ivfpq import IvfPqIndex
    m = H.ivfpq_tie_model()
    single = IvfPqIndex("euclidean", 64, m["cent"], m["cb"], nprobe=8)
    single.add(m["base"], m["asg"], m["codes"])
    for k in (10, 20):
        d_ref, r_ref = single.search_batch(m["queries"], k)
        assert np.array_equal(got[f"rows{k}"], r_ref)
        assert np.array_equal(got[f"dist{k}"].view(np.uint32), d_ref.view(np.uint32))
