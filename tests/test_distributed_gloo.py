"""Multi-process host logic of the row-sharded search, on CPU with gloo ranks
(world sizes 2 and 3): contiguous row ranges as split_ids
(GpuDistributedIndex.cpp:12-22), global row offsets, the rank-major candidate
exchange, and the root's merge, checked against the unsharded search. Each
rank's local top-k comes from the oracle here (the per-shard device search is
covered by the GPU tests); the exchange is the product's. Also: a rank that
never joins makes the others' exchange end with an error within the process
group's short timeout instead of hanging."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import oracle as O
from elips_b200.distributed import exchange_candidates, shard_range
from tests import helpers as H


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


CASES = [("euclidean", 3000), ("cosine", 2999), ("euclidean", 5), ("dot_product", 1000)]


def _case_data(metric, n):
    base = H.gaussian(n, 16, seed=71 + n)
    queries = H.gaussian(7, 16, seed=72)
    if metric == "cosine":
        base, queries = H.normalize(base), H.normalize(queries)
    return base, queries


def _worker(rank, world, port, k, out_dir):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        for c, (metric, n) in enumerate(CASES):
            base, queries = _case_data(metric, n)
            lo, hi = shard_range(base.shape[0], rank, world)
            d, r = O.exact_search(metric, base[lo:hi], queries, k, 1)
            # candidate block: (distance bits, global row); absent entries keep row -1
            block = torch.empty((queries.shape[0], k, 2), dtype=torch.int64)
            block[..., 0] = torch.from_numpy(d.view(np.int32).astype(np.int64))
            block[..., 1] = torch.from_numpy(np.where(r >= 0, r + lo, -1))
            gathered = exchange_candidates(block, world).numpy()
            if rank == 0:
                np.save(os.path.join(out_dir, f"gathered{c}.npy"), gathered)
    finally:
        dist.destroy_process_group()


def _merge(gathered, k):
    """Root merge: k smallest by (distance, row) over the rank-major blocks."""
    world, nq = gathered.shape[:2]
    dist = gathered[..., 0].astype(np.int32).view(np.float32)
    rows = gathered[..., 1]
    out_d = np.zeros((nq, k), np.float32)
    out_r = np.full((nq, k), -1, np.int64)
    for q in range(nq):
        dq = dist[:, q].reshape(-1)
        rq = rows[:, q].reshape(-1)
        keep = rq >= 0
        order = np.lexsort((rq[keep], dq[keep]))[:k]
        out_d[q, :len(order)] = dq[keep][order]
        out_r[q, :len(order)] = rq[keep][order]
    return out_d, out_r


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_exchange_matches_unsharded_search(tmp_path, world):
    k = 4
    mp.spawn(_worker, args=(world, _free_port(), k, str(tmp_path)), nprocs=world, join=True)
    for c, (metric, n) in enumerate(CASES):
        base, queries = _case_data(metric, n)
        d, r = _merge(np.load(tmp_path / f"gathered{c}.npy"), k)
        d_ref, r_ref = O.exact_search(metric, base, queries, k, 1)
        assert np.array_equal(r, r_ref) and np.array_equal(d, d_ref), (metric, n)


def test_shard_ranges_partition_the_rows():
    for n in (0, 1, 7, 1000, 2_000_000):
        for world in (1, 2, 3, 8):
            spans = [shard_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            assert max(b - a for a, b in spans) - min(b - a for a, b in spans) <= 1


def _absent_rank_worker(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        return  # leaves between steps: never joins the exchange
    try:
        exchange_candidates(torch.zeros((2, 3, 2), dtype=torch.int64), world)
        outcome = "completed"
    except Exception as e:  # the short process-group timeout or the closed peer
        outcome = "error: " + type(e).__name__
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(outcome)


def test_absent_rank_fails_the_exchange_instead_of_hanging(tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_absent_rank_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert (tmp_path / "rank0.txt").read_text().startswith("error")


def test_balanced_lists_partition():
    from elips_b200.distributed import balanced_lists
    rng = np.random.default_rng(5)
    sizes = rng.integers(0, 5000, 4096)
    for world in (1, 2, 3, 8):
        owner = balanced_lists(sizes, world)
        assert owner.shape == sizes.shape and set(owner.tolist()) <= set(range(world))
        load = np.bincount(owner, weights=sizes.astype(float) ** 2, minlength=world)
        assert load.max() <= load.mean() + (sizes.astype(float) ** 2).max()
        assert np.array_equal(owner, balanced_lists(sizes, world))
        # item-aware weights: ceil(count / G) items, each costing size + item_rows
        counts = rng.integers(0, 200, sizes.size)
        owner = balanced_lists(sizes, world, counts, queries_per_item=8, item_rows=1024)
        w = np.ceil(counts / 8) * np.where(sizes > 0, sizes + 1024.0, 0.0)
        load = np.bincount(owner, weights=w, minlength=world)
        assert load.max() <= load.mean() + w.max()


def _probe_worker(rank, world, port, out_dir):
    """Each rank probes its slice of the batch (the oracle stands in for the
    device probe), the padded slices go through the product's exchange, and
    the product's probe_table reassembles the full table."""
    import torch
    import torch.distributed as dist
    from elips_b200.distributed import ShardedIvfPqIndex
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        for nq in (1, 7, 50):
            cents = H.gaussian(40, 12, seed=91)
            q = H.gaussian(nq, 12, seed=92 + nq)
            lo, hi, chunk = ShardedIvfPqIndex.probe_rows(nq, rank, world)
            block = torch.zeros((chunk, 5), dtype=torch.int32)
            if hi > lo:
                block[:hi - lo] = torch.from_numpy(O.ivf_probe("euclidean", q[lo:hi], cents, 5).view(np.int32))
            table = ShardedIvfPqIndex.probe_table(exchange_candidates(block, world), nq).numpy()
            if rank == 0:
                np.save(os.path.join(out_dir, f"probes{nq}.npy"), table)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_split_probe_exchange_equals_full_probe(tmp_path, world):
    """The IVF-PQ probe split across ranks (ShardedIvfPqIndex.probe_rows /
    probe_table over exchange_candidates) gives the full batch's probe table,
    including batches smaller than the world (empty, padded slices)."""
    mp.spawn(_probe_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for nq in (1, 7, 50):
        cents = H.gaussian(40, 12, seed=91)
        q = H.gaussian(nq, 12, seed=92 + nq)
        got = np.load(tmp_path / f"probes{nq}.npy")
        assert np.array_equal(got.view(np.uint32), O.ivf_probe("euclidean", q, cents, 5))


class _OracleReplica:
    """A replica whose per-slice search is the oracle's (CPU tensors in and
    out); the split of the batch and the all-gather are the product's."""

    def __init__(self, metric, base):
        self.metric, self.base = metric, base

    def size(self):
        return self.base.shape[0]

    def search_device(self, queries, k):
        import torch
        d, r = O.exact_search(self.metric, self.base, queries.numpy(), k, 1)
        return torch.from_numpy(d), torch.from_numpy(r.astype(np.int64))


def _replica_worker(rank, world, port, k, out_dir):
    import torch
    import torch.distributed as dist
    from elips_b200.distributed import ReplicatedIndex
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        for c, (metric, n) in enumerate(CASES):
            base, queries = _case_data(metric, n)
            index = ReplicatedIndex(_OracleReplica(metric, base))
            assert index.size() == n and index.type_name() == "gpu_replicated"
            for nq in (7, 2, 1, 0):
                d, r = index.search_device(torch.from_numpy(queries[:nq]), k)
                np.save(os.path.join(out_dir, f"rep{c}_{nq}_r{rank}_d.npy"), d.numpy())
                np.save(os.path.join(out_dir, f"rep{c}_{nq}_r{rank}_r.npy"), r.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_replicated_query_split_matches_one_replica(tmp_path, world):
    """DistributedMode::replicate: every rank answers its query_range slice of
    the batch against a full replica; after the all-gather every rank holds
    the whole batch's results in query order, equal to one replica's answer
    for the whole batch (batches smaller than the world leave ranks idle)."""
    k = 4
    mp.spawn(_replica_worker, args=(world, _free_port(), k, str(tmp_path)), nprocs=world, join=True)
    for c, (metric, n) in enumerate(CASES):
        base, queries = _case_data(metric, n)
        for nq in (7, 2, 1, 0):
            d_ref, r_ref = O.exact_search(metric, base, queries[:nq], k, 1)
            for rank in range(world):
                d = np.load(tmp_path / f"rep{c}_{nq}_r{rank}_d.npy")
                r = np.load(tmp_path / f"rep{c}_{nq}_r{rank}_r.npy")
                assert d.shape == (nq, k) and r.shape == (nq, k)
                assert np.array_equal(r, r_ref) and np.array_equal(d.view(np.uint32), d_ref.view(np.uint32))


def test_query_ranges_partition_the_batch():
    from elips_b200.distributed import query_range
    for nq in (0, 1, 5, 10_000):
        for world in (1, 2, 3, 8):
            spans = [query_range(nq, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == nq
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))


def test_shard_candidates_global_rows():
    import torch
    from elips_b200.distributed import shard_candidates
    d = torch.tensor([[0.5, 1.25, float("inf")]], dtype=torch.float32)
    r = torch.tensor([[3, 0, -1]], dtype=torch.int64)
    c = shard_candidates(d, r, 1000)
    assert c.dtype == torch.int32 and c.shape == (1, 3, 2)
    assert c[0, :, 1].tolist() == [1003, 1000, -1]
    assert torch.equal(c[..., 0], d.view(torch.int32))


def test_slice_mask_rebases_each_rank():
    """The filter of a row-sharded filtered search: a rank's mask is the global
    mask's bits for its rows, its first row at bit 0 (ragged ranges, ranges
    not starting on a word boundary, empty ranges)."""
    from elips_b200.distributed import slice_mask
    rng = np.random.default_rng(7)
    for n in (0, 1, 33, 1000, 4099):
        bits = rng.random(n) < 0.3
        words = np.zeros((n + 31) // 32, np.uint32)
        for i in np.flatnonzero(bits):
            words[i >> 5] |= np.uint32(1) << np.uint32(i & 31)
        for world in (1, 2, 3, 8):
            for rank in range(world):
                lo, hi = shard_range(n, rank, world)
                sub = slice_mask(words, lo, hi)
                assert sub.shape == ((hi - lo + 31) // 32,)
                got = [(int(sub[j >> 5]) >> (j & 31)) & 1 for j in range(hi - lo)]
                assert got == bits[lo:hi].astype(int).tolist()


def test_peer_set_layout_keeps_every_part_aligned():
    """The root's exchange buffer holds two sets of (candidate blocks, bounds);
    with odd batch sizes (a single query) the second set and the bounds must
    still start on 256 bytes, or the merge kernel's 8-byte loads of the second
    set fault."""
    from elips_b200.distributed import peer_set_layout
    for world in (2, 3, 8):
        for nq in (1, 3, 7, 8, 63, 64, 500, 10_000):
            for k in (1, 10, 20, 100):
                recv, set_bytes = peer_set_layout(world, nq, k)
                assert recv % 256 == 0 and set_bytes % 256 == 0
                assert recv >= world * nq * k * 8 and set_bytes >= recv + nq * 4
