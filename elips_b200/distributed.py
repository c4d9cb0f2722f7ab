"""Row-sharded exact search over the GPUs of one node, one process per GPU.

Mirrors GpuDistributedIndex in shard mode (src/gpu_engine/GpuDistributedIndex.cpp):
the base set is split into contiguous row ranges exactly as split_ids does
(:12-22, rows [N*s/S, N*(s+1)/S)), every rank searches its own range with the
fused tensor-core kernel, and the per-rank top-k lists are merged. Where the
reference loops over its shards on the host and merges with partial_sort
(:68-83, :155-207), here each rank writes its k candidates (ordering key,
global row) on its own GPU, one NCCL all-gather over NVLink moves them, and
the final top-k kernel merges them on the root rank.

torch.distributed (backend "nccl") is the plumbing; the search and the merge
are the library's kernels behind the C ABI.
"""
from __future__ import annotations

from typing import Optional

import numpy as np

from .exact import ExactIndex, merge_candidates_device


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """split_ids (GpuDistributedIndex.cpp:12-22): [n*rank/world, n*(rank+1)/world)."""
    return n * rank // world, n * (rank + 1) // world


def exchange_candidates(cand, world: int, group=None):
    """All-gather of every rank's candidate block [nq, k, ...] into
    [world, nq, k, ...], rank-major (rank r's block at index r). The output is
    gathered flat, which every backend accepts: NCCL over NVLink for CUDA
    tensors, gloo for CPU tensors. Collective: every rank of the group calls
    it with blocks of the same shape."""
    import torch
    import torch.distributed as dist
    cand = cand.contiguous()
    flat = torch.empty((world * cand.shape[0],) + tuple(cand.shape[1:]), dtype=cand.dtype, device=cand.device)
    dist.all_gather_into_tensor(flat, cand, group=group)
    return flat.view((world,) + tuple(cand.shape))


class ShardedExactIndex:
    """One rank's share of a row-sharded index. Every rank of the process group
    must call each method with the same arguments (collective semantics)."""

    def __init__(self, metric: str, dimension: int, total_rows: int, precision: str = "fp16",
                 device: Optional[int] = None, group=None):
        import torch
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.device = torch.cuda.current_device() if device is None else device
        self.metric = metric
        self.dimension = dimension
        self.total_rows = total_rows
        self.row_begin, self.row_end = shard_range(total_rows, self.rank, self.world)
        self.local = ExactIndex(metric, dimension, precision=precision, device=self.device)

    def add_device(self, rows) -> None:
        """Appends this rank's rows (a CUDA tensor); rows must arrive in global order."""
        self.local.add_device(rows)

    def search_device(self, queries, k: int, mask=None):
        """queries: CUDA tensor on every rank (same values). Returns (dist, rows)
        CUDA tensors on the root rank, (None, None) elsewhere."""
        import torch
        nq = queries.shape[0]
        dev = queries.device
        if self.world == 1:
            return self.local.search_device(queries, k, mask=mask)
        cand = torch.empty((nq, k, 2), dtype=torch.int32, device=dev)
        self.local.search_candidates_device(queries, k, self.row_begin, cand, mask=mask)
        gathered = exchange_candidates(cand, self.world, self.group)
        if self.rank != 0:
            return None, None
        return merge_candidates_device(gathered, self.world, k, self.metric)

    def search_batch(self, queries_host, k: int, out_dist=None, out_rows=None):
        """End-to-end search from host memory: uploads the queries on every rank,
        searches, gathers, merges, and copies the k results back to host memory on
        the root rank. queries_host: pinned CPU torch tensor (or numpy array)."""
        import torch
        q = torch.as_tensor(queries_host)
        qd = q.to(f"cuda:{self.device}", non_blocking=True)
        d, r = self.search_device(qd, k)
        if d is None:
            return None, None
        if out_dist is None:
            out_dist = torch.empty(d.shape, dtype=d.dtype, pin_memory=True)
            out_rows = torch.empty(r.shape, dtype=r.dtype, pin_memory=True)
        out_dist.copy_(d, non_blocking=True)
        out_rows.copy_(r, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return out_dist, out_rows
