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

from .exact import METRICS as METRICS_CODE
from .exact import ExactIndex, merge_candidates_device


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """split_ids (GpuDistributedIndex.cpp:12-22): [n*rank/world, n*(rank+1)/world)."""
    return n * rank // world, n * (rank + 1) // world


def slice_mask(words, lo: int, hi: int) -> np.ndarray:
    """A global eligibility mask (uint32 words, bit i & 31 of word i >> 5 =
    row i) cut to the rows [lo, hi) a rank holds, re-based so the rank's first
    row is bit 0: the filter of a row-sharded filtered search."""
    words = np.asarray(words, np.uint32)
    out = np.zeros((hi - lo + 31) // 32, np.uint32)
    if hi <= lo:
        return out
    idx = np.arange(lo, hi)
    on = np.nonzero((words[idx >> 5] >> (idx & 31).astype(np.uint32)) & 1)[0]
    np.bitwise_or.at(out, on >> 5, np.left_shift(np.uint32(1), (on & 31).astype(np.uint32)))
    return out


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


def peer_set_layout(world: int, nq: int, k: int) -> tuple[int, int]:
    """(bytes before the bounds, bytes of one buffer set) of PeerExchange's
    root buffer: the candidate blocks (world x nq x k pairs of 8 bytes), then
    nq 4-byte bounds, each part rounded up to 256 bytes so that the second
    set, the bounds and every block start aligned whatever nq is (the merge
    kernel reads the blocks with 8- and 16-byte loads)."""
    def up(x):
        return (x + 255) // 256 * 256
    recv = up(world * nq * k * 8)
    return recv, up(recv + nq * 4)


class PeerExchange:
    """The shard exchange over NVLink peer memory (one process per GPU of one
    node): the root owns, twice over (alternating steps), a receive buffer for
    every rank's [nq, k] candidate block and nq shared per-query admission
    bounds; every rank maps them (CUDA interprocess handles) and
      * passes the bounds to its fused kernel, which reads and tightens them
        while it runs, so a shard admits only candidates that can still reach
        the global top-k;
      * copies its k candidates per query straight into its slot of the
        root's buffer (a device-to-peer copy), where the root's merge kernel
        reads them after one tiny all-reduce orders the ranks.
    Collective: every rank calls ensure() and step() in the same order."""

    def __init__(self, rank: int, world: int, device: int, group=None):
        import torch
        import torch.distributed as dist
        self.dist, self.group = dist, group
        self.rank, self.world, self.device = rank, world, device
        self.cap_q = self.k = 0
        self.base = None         # this process's mapping of the root's buffer
        self.owned = None        # the root's own allocation
        self.step_no = 0
        self.flag = torch.zeros(1, dtype=torch.int32, device=f"cuda:{device}")

    def _sizes(self, nq, k):
        return peer_set_layout(self.world, nq, k)

    def ensure(self, nq: int, k: int) -> None:
        """(Re)creates the buffers for batches of up to nq queries at this k."""
        import ctypes
        from . import _capi as capi
        if nq <= self.cap_q and k == self.k:
            return
        self.close()
        cap_q = max(nq, self.cap_q)
        _, set_bytes = self._sizes(cap_q, k)
        handle = (ctypes.c_uint8 * 64)()
        if self.rank == 0:
            ptr = ctypes.c_void_p()
            capi.check(capi.LIB.elips_b200_peer_alloc(self.device, 2 * set_bytes, ctypes.byref(ptr), handle),
                       "elips_b200_peer_alloc")
            self.owned = self.base = ptr.value
            capi.check(capi.LIB.elips_b200_fill_device(self.device, self.base, 0xFF, 2 * set_bytes, None),
                       "elips_b200_fill_device")
            import torch
            torch.cuda.synchronize(self.device)
        obj = [bytes(handle)]
        self.dist.broadcast_object_list(obj, src=0, group=self.group)
        if self.rank != 0:
            ctypes.memmove(handle, obj[0], 64)
            ptr = ctypes.c_void_p()
            capi.check(capi.LIB.elips_b200_peer_open(self.device, handle, ctypes.byref(ptr)), "elips_b200_peer_open")
            self.base = ptr.value
        self.cap_q, self.k = cap_q, k
        self.dist.barrier(group=self.group)

    def slots(self, nq: int):
        """(this rank's candidate slot, the bounds, the root's candidate
        blocks) of the current step's buffer set, as device addresses."""
        _, set_bytes = self._sizes(self.cap_q, self.k)
        recv_bytes, _ = self._sizes(self.cap_q, self.k)
        s = self.base + (self.step_no & 1) * set_bytes
        return s + self.rank * nq * self.k * 8, s + recv_bytes, s

    def finish_step(self, nq: int, stream) -> None:
        """Root: resets the other set's bounds for the next step; all: one
        all-reduce that orders every rank's copy before the root's merge."""
        from . import _capi as capi
        if self.rank == 0:
            _, set_bytes = self._sizes(self.cap_q, self.k)
            recv_bytes, _ = self._sizes(self.cap_q, self.k)
            other = self.base + ((self.step_no + 1) & 1) * set_bytes + recv_bytes
            # every bound of the set: the next step may carry more queries
            capi.check(capi.LIB.elips_b200_fill_device(self.device, other, 0xFF, self.cap_q * 4, stream),
                       "elips_b200_fill_device")
        self.dist.all_reduce(self.flag, group=self.group)
        self.step_no += 1

    def close(self) -> None:
        """Collective: the other ranks unmap the root's buffer, then the root frees it."""
        import torch
        from . import _capi as capi
        if self.base is None:
            return
        torch.cuda.synchronize(self.device)
        if self.rank != 0:
            capi.LIB.elips_b200_peer_close(self.device, self.base)
        self.dist.barrier(group=self.group)
        if self.owned is not None:
            capi.LIB.elips_b200_peer_free(self.device, self.owned)
        self.base = self.owned = None
        self.cap_q = self.k = 0


class ShardedExactIndex:
    """One rank's share of a row-sharded index. Every rank of the process group
    must call each method with the same arguments (collective semantics).

    exchange="peer" (default with NCCL): the ranks share their admission
    bounds while their kernels run and hand their candidates to the root over
    NVLink peer memory (PeerExchange); "allgather": private bounds and an NCCL
    all-gather of the candidate blocks (any backend)."""

    def __init__(self, metric: str, dimension: int, total_rows: int, precision: str = "fp16",
                 device: Optional[int] = None, group=None, exchange: Optional[str] = None):
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
        if exchange is None:
            exchange = "peer" if (self.world > 1 and dist.get_backend(group) == "nccl") else "allgather"
        self.exchange = exchange
        self.peer = PeerExchange(self.rank, self.world, self.device, group) if exchange == "peer" else None

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
        if self.peer is not None:
            return self._search_peer(queries, k, mask, cand)
        self.local.search_candidates_device(queries, k, self.row_begin, cand, mask=mask)
        gathered = exchange_candidates(cand, self.world, self.group)
        if self.rank != 0:
            return None, None
        return merge_candidates_device(gathered, self.world, k, self.metric)

    def _search_peer(self, queries, k, mask, cand):
        import torch
        from . import _capi as capi
        nq = queries.shape[0]
        self.peer.ensure(nq, k)
        my_slot, bounds, blocks = self.peer.slots(nq)
        stream = torch.cuda.current_stream(queries.device).cuda_stream
        capi.check(capi.LIB.elips_b200_exact_search_candidates_shared_device(
            self.local._h, queries.data_ptr(), nq, k, mask.data_ptr() if mask is not None else None,
            self.row_begin, cand.data_ptr(), bounds, stream), "elips_b200_exact_search_candidates_shared_device")
        capi.check(capi.LIB.elips_b200_copy_device(self.device, my_slot, cand.data_ptr(), nq * k * 8, stream),
                   "elips_b200_copy_device")
        self.peer.finish_step(nq, stream)
        if self.rank != 0:
            return None, None
        out_dist = torch.empty((nq, k), dtype=torch.float32, device=queries.device)
        out_rows = torch.empty((nq, k), dtype=torch.int64, device=queries.device)
        capi.check(capi.LIB.elips_b200_merge_candidates_device(
            self.device, blocks, nq, self.world, k, METRICS_CODE[self.metric], out_dist.data_ptr(),
            out_rows.data_ptr(), stream), "elips_b200_merge_candidates_device")
        return out_dist, out_rows

    def search_batch(self, queries_host, k: int, out_dist=None, out_rows=None, mask=None):
        """End-to-end search from host memory: uploads the queries on every rank,
        searches, gathers, merges, and copies the k results back to host memory on
        the root rank. queries_host: pinned CPU torch tensor (or numpy array).
        mask: this rank's row filter as host uint32 words (slice_mask of the
        global filter), uploaded with the queries."""
        import torch
        q = torch.as_tensor(queries_host)
        qd = q.to(f"cuda:{self.device}", non_blocking=True)
        md = None
        if mask is not None:
            md = torch.from_numpy(np.ascontiguousarray(mask, np.uint32).view(np.int32)).to(
                f"cuda:{self.device}", non_blocking=True)
        d, r = self.search_device(qd, k, mask=md)
        if d is None:
            return None, None
        if out_dist is None:
            out_dist = torch.empty(d.shape, dtype=d.dtype, pin_memory=True)
            out_rows = torch.empty(r.shape, dtype=r.dtype, pin_memory=True)
        out_dist.copy_(d, non_blocking=True)
        out_rows.copy_(r, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return out_dist, out_rows


def shard_candidates(dist, rows, row_begin: int):
    """One shard's results (dist [nq, k] float32, local rows [nq, k] int64,
    -1 = none) as [nq, k, 2] int32 candidate pairs (distance bits, global
    row = row_begin + local row), the block exchange_candidates moves."""
    import torch
    glob = torch.where(rows >= 0, rows + row_begin, rows)
    return _pairs(dist, glob)


class ShardedRowsIndex:
    """Row sharding (split_ids ranges, GpuDistributedIndex.cpp:12-22) over any
    per-rank index whose search_device returns final distances and local
    rows: the quantized ExactIndex (QuantizedIndex, sq8 / PQ / OPQ codes) is
    the one that needs it, the exact index has the fused ShardedExactIndex.
    Each rank searches the rows it holds, its k results become (distance,
    global row) pairs, one all-gather moves them and the root's merge kernel
    keeps the k smallest by (distance, row), the order one index over all
    rows returns. The distances are final, so the merge applies no transform.
    Every rank of the group must call search_device with the same batch."""

    def __init__(self, local, total_rows: int, group=None):
        import torch.distributed as dist
        self.local = local
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.total_rows = total_rows
        self.row_begin, self.row_end = shard_range(total_rows, self.rank, self.world)

    def search_device(self, queries, k: int):
        """queries: CUDA tensor, the same batch on every rank. Returns (dist,
        global rows) CUDA tensors on the root rank, (None, None) elsewhere."""
        d, r = self.local.search_device(queries, k)
        if self.world == 1:
            return d, r
        gathered = exchange_candidates(shard_candidates(d, r, self.row_begin), self.world, self.group)
        if self.rank != 0:
            return None, None
        return merge_candidates_device(gathered, self.world, k, "dot_product")


def query_range(nq: int, rank: int, world: int) -> tuple[int, int]:
    """The slice of a query batch one replica answers: contiguous, split as
    split_ids splits rows (GpuDistributedIndex.cpp:12-22)."""
    return nq * rank // world, nq * (rank + 1) // world


def gather_query_slices(dist_slice, rows_slice, nq: int, world: int, group=None):
    """All-gather of every rank's results for its query_range slice into the
    whole batch's (dist [nq, k] float32, rows [nq, k] int64), in query order,
    on every rank. Slices are padded to ceil(nq / world) queries so the
    collective moves equal blocks; (distance bits, row low, row high) travel
    as one int32 block. Collective: every rank calls it with the same nq."""
    import torch
    import torch.distributed as dist
    k = dist_slice.shape[1]
    per = (nq + world - 1) // world
    dev = dist_slice.device
    if per == 0:
        return (torch.empty((0, k), dtype=torch.float32, device=dev),
                torch.empty((0, k), dtype=torch.int64, device=dev))
    m = dist_slice.shape[0]
    block = torch.empty((per, k, 3), dtype=torch.int32, device=dev)
    block[:m, :, 0] = dist_slice.contiguous().view(torch.int32)
    block[:m, :, 1:] = rows_slice.contiguous().view(torch.int32).view(m, k, 2)
    flat = torch.empty((world * per, k, 3), dtype=torch.int32, device=dev)
    dist.all_gather_into_tensor(flat, block, group=group)
    take = torch.cat([torch.arange(r * per, r * per + (query_range(nq, r, world)[1] - query_range(nq, r, world)[0]))
                      for r in range(world)]).to(dev)
    g = flat.index_select(0, take)
    return g[..., 0].contiguous().view(torch.float32), g[..., 1:].contiguous().view(torch.int64).view(nq, k)


class ReplicatedIndex:
    """GpuDistributedIndex in replicate mode (DistributedMode::replicate,
    src/gpu_engine/GpuDistributedIndex.cpp): every rank holds a full copy of
    the index. Inserts go to every replica (:50-55), removals too (:61-65),
    and the size is one replica's (:110-112). For a batch the reference hands
    the whole batch to one replica in turn (:173-177); here the batch is split
    across the replicas by contiguous query ranges and the slices are
    all-gathered, so one batch keeps every GPU busy and no base row crosses
    NVLink. A query's results do not depend on which other queries share its
    launch, so they equal one replica's answer for the whole batch.

    `local` is this rank's index (ExactIndex, IvfPqIndex or IvfFlatIndex) on
    its own GPU; every rank must build it from the same rows in the same order
    and call search_device / search_batch with the same batch size."""

    def __init__(self, local, group=None):
        import torch.distributed as dist
        self.local = local
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1

    def type_name(self) -> str:
        """GpuDistributedIndex::type_name (:116-118)."""
        return "gpu_replicated"

    def size(self) -> int:
        return self.local.size()

    def add_device(self, rows, *args) -> None:
        """Appends the same rows to this replica (every rank does)."""
        self.local.add_device(rows, *args)

    def remove(self, slot: int):
        return self.local.remove(slot)

    def search_device(self, queries, k: int, **kwargs):
        """queries: CUDA tensor [nq, d], the same batch on every rank. This rank
        answers query_range(nq, rank, world); returns the whole batch's
        (dist, rows) on every rank."""
        import torch
        nq = queries.shape[0]
        lo, hi = query_range(nq, self.rank, self.world)
        if hi > lo:
            d, r = self.local.search_device(queries[lo:hi], k, **kwargs)
        else:
            d = torch.empty((0, k), dtype=torch.float32, device=queries.device)
            r = torch.empty((0, k), dtype=torch.int64, device=queries.device)
        if self.world == 1:
            return d, r
        return gather_query_slices(d, r, nq, self.world, self.group)

    def search_batch(self, queries_host, k: int, out_dist=None, out_rows=None, device=None):
        """End-to-end from host memory: every rank uploads only its own slice of
        the batch, searches it, the slices are all-gathered, and the root copies
        the whole batch's results to host memory (other ranks return None, None)."""
        import torch
        q = torch.as_tensor(queries_host)
        nq = q.shape[0]
        dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        lo, hi = query_range(nq, self.rank, self.world)
        per = (nq + self.world - 1) // self.world
        if hi > lo:
            d, r = self.local.search_device(q[lo:hi].to(dev, non_blocking=True), k)
        else:
            d = torch.empty((0, k), dtype=torch.float32, device=dev)
            r = torch.empty((0, k), dtype=torch.int64, device=dev)
        if self.world > 1 and per > 0:
            d, r = gather_query_slices(d, r, nq, self.world, self.group)
        if self.rank != 0:
            return None, None
        if out_dist is None:
            out_dist = torch.empty((nq, k), dtype=torch.float32, pin_memory=True)
            out_rows = torch.empty((nq, k), dtype=torch.int64, pin_memory=True)
        out_dist.copy_(d, non_blocking=True)
        out_rows.copy_(r, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
        return out_dist, out_rows


def list_range(nlist: int, rank: int, world: int) -> tuple[int, int]:
    """The IVF lists a rank owns: contiguous list ids, split as split_ids splits
    rows (GpuDistributedIndex.cpp:12-22)."""
    return nlist * rank // world, nlist * (rank + 1) // world


def balanced_lists(list_sizes, world: int, probe_counts=None, queries_per_item: int = 0,
                   item_rows: int = 1024) -> np.ndarray:
    """Owner rank of every IVF list, balancing the scan work: a probed list
    costs its size times the queries that probe it. With `probe_counts` (how
    often each list was probed by a sample of queries) the weight is
    size x count; without it, queries are taken to probe lists about in
    proportion to their size and the weight is size^2. With
    `queries_per_item` (the scan's group size G: a scan item streams a list
    once for up to G of its queries, and costs the same for fewer) the weight
    is ceil(count / G) x (size + item_rows), item_rows standing for an item's
    fixed cost (its lookup tables, start and write-out) in list rows.
    Greedy longest-first: heaviest list to the least loaded rank (ties: lower
    list id, lower rank). Deterministic, so every rank computes the same
    partition."""
    sizes = np.asarray(list_sizes, np.float64)
    if probe_counts is not None and queries_per_item > 0:
        items = np.ceil(np.asarray(probe_counts, np.float64) / queries_per_item)
        weight = items * np.where(sizes > 0, sizes + item_rows, 0.0)
    else:
        weight = sizes * (sizes if probe_counts is None else np.asarray(probe_counts, np.float64))
    order = np.lexsort((np.arange(sizes.size), -weight))
    load = np.zeros(world)
    owner = np.empty(sizes.size, np.int64)
    for l in order:
        r = int(np.argmin(load))
        owner[l] = r
        load[r] += weight[l]
    return owner


def _pairs(dist, rows):
    """(dist [nq, m] float32, rows [nq, m] int64, -1 = none) -> [nq, m, 2] int32
    candidate pairs (distance bits, row)."""
    import torch
    return torch.stack((dist.contiguous().view(torch.int32), rows.to(torch.int32)), dim=-1)


class ShardedIvfPqIndex:
    """One rank's share of a list-sharded IVF-PQ index. The reference shards
    rows in GpuDistributedIndex and retrains a model per shard (:318-320);
    here every rank holds the one global model and the ranks together answer
    exactly what a single index answers.

    Rank r owns the lists that `owner` (one rank per list, e.g. balanced_lists
    of the global list sizes) gives it, by default list_range(nlist, r, world),
    and only their rows. A search
    (every rank calls it with the same queries):
      1. each rank: probe (replicated centroids), scan its own probed lists,
         R = 4k best approximate (distance, global slot);
      2. all-gather; every rank merges the R best over all ranks, the set a
         single index would rerank;
      3. each rank reranks the ones it holds, exactly, on its raw rows;
      4. all-gather of the k best per rank; the root merges them by
         (distance, global slot).
    Before step 1 the probe itself is split: each rank probes a slice of the
    batch and the slices are exchanged (probe_slice, probe_table).
    The phases are methods, so a test can drive several ranks in one process;
    `exchange` defaults to exchange_candidates over the process group.

    With a PeerExchange (`peer`; made by default for NCCL process groups
    when `exchange` is not given) the ranks' scans share their per-query
    admission bounds through the root's memory while they run (a bound any
    rank publishes is the R-th key of R of its candidates, so no candidate of
    the global R best is dropped), and step 4 becomes a copy of each rank's
    k best into its slot of the root's buffer plus one 4-byte all-reduce."""

    def __init__(self, metric: str, dimension: int, centroids, codebook, nprobe: int, pq_bits: int = 8,
                 rank: int = 0, world: int = 1, device: int = 0, group=None, exchange=None, owner=None,
                 peer=None):
        import torch
        from .ivfpq import IvfPqIndex
        self.metric, self.rank, self.world, self.group = metric, rank, world, group
        self.nlist = np.asarray(centroids).shape[0]
        if owner is None:
            owner = np.empty(self.nlist, np.int64)
            for r in range(world):
                lo, hi = list_range(self.nlist, r, world)
                owner[lo:hi] = r
        owned = np.asarray(owner) == rank
        self.local = IvfPqIndex(metric, dimension, centroids, codebook, nprobe=nprobe, pq_bits=pq_bits,
                                device=device)
        self.local.set_owned_lists(owned)
        self.owned = torch.from_numpy(owned).to(f"cuda:{device}")
        self.global_rows = None  # int64 device tensor, ascending: local slot -> global slot
        self._local_of = None    # int32 device tensor: global slot -> local slot or -1
        if peer is None and exchange is None and world > 1:
            import torch.distributed as dist
            if dist.is_initialized() and dist.get_backend(group) == "nccl":
                peer = PeerExchange(rank, world, device, group)
        self.peer = peer or None   # peer=False: NCCL all-gathers only
        self.exchange = exchange if exchange is not None else (
            lambda t: exchange_candidates(t, self.world, self.group))

    def close(self) -> None:
        """Collective: releases the peer buffers (every rank calls it)."""
        if self.peer is not None:
            self.peer.close()

    def add_device(self, vectors, assignments, first_row: int, codes=None) -> None:
        """Offers rows [first_row, first_row + n) in global order (CUDA tensors;
        assignments int32); this rank keeps those of its own lists."""
        import torch
        idx = torch.nonzero(self.owned[assignments.long()]).flatten()
        if idx.numel() == 0:
            return
        self.local.add_device(vectors[idx].contiguous(), assignments[idx].contiguous(),
                              None if codes is None else codes[idx].contiguous())
        g = idx + first_row
        self.global_rows = g if self.global_rows is None else torch.cat((self.global_rows, g))
        self._local_of = None

    def _to_global(self, rows):
        import torch
        if self.global_rows is None:
            return torch.full_like(rows, -1)
        return torch.where(rows >= 0, self.global_rows[rows.clamp(min=0)], rows)

    def _to_local(self, rows):
        """Global slots -> this rank's slots (-1: none, or held by another
        rank), through a dense map over the global slots built once per
        change of the rows."""
        import torch
        if self.global_rows is None:
            return torch.full_like(rows, -1)
        if self._local_of is None:
            top = int(self.global_rows.max().item()) + 1
            self._local_of = torch.full((top + 1,), -1, dtype=torch.int32, device=self.global_rows.device)
            self._local_of[self.global_rows] = torch.arange(self.global_rows.numel(), dtype=torch.int32,
                                                            device=self.global_rows.device)
        top = self._local_of.numel() - 1           # the last entry stays -1: rows past this rank's last
        return self._local_of[rows.clamp(min=0, max=top)].long().masked_fill_(rows < 0, -1)

    @staticmethod
    def probe_rows(nq: int, rank: int, world: int) -> tuple[int, int, int]:
        """(lo, hi, chunk): the queries [lo, hi) rank probes, every rank's block
        padded to chunk = ceil(nq / world) rows (equal shapes for the exchange)."""
        chunk = (nq + world - 1) // world
        return min(nq, rank * chunk), min(nq, (rank + 1) * chunk), chunk

    def probe_slice(self, queries):
        """Phase 0: this rank's slice of the probe, padded to ceil(nq / world)
        rows so that every rank's block has the same shape: [chunk, nprobe] int32."""
        import torch
        nq = queries.shape[0]
        lo, hi, chunk = self.probe_rows(nq, self.rank, self.world)
        out = torch.zeros((chunk, min(self.local.nprobe, self.nlist)), dtype=torch.int32, device=queries.device)
        if hi > lo:
            out[:hi - lo] = self.local.probe_device(queries[lo:hi].contiguous())
        return out

    @staticmethod
    def probe_table(gathered, nq: int):
        """The full probe table from the gathered slices [world, chunk, nprobe]."""
        return gathered.reshape(-1, gathered.shape[-1])[:nq].contiguous()

    def approx_candidates(self, queries, k: int, probes=None, shared_bound=None):
        """Phase 1: [nq, 4k, 2] int32 (distance bits, global slot). `probes`
        (the full [nq, nprobe] table, e.g. from probe_slice + exchange) skips
        this rank's own probe of the whole batch; `shared_bound` (device
        address of nq bounds shared by the ranks) replaces the scan's own."""
        import torch
        cand = self.local.search_candidates_device(queries, k, probes=probes, shared_bound=shared_bound)
        return _pairs(cand[..., 0].contiguous().view(torch.float32), self._to_global(cand[..., 1].long()))

    def rerank_owned(self, queries, k: int, gathered):
        """Phases 2-3: gathered [world, nq, 4k, 2] -> this rank's [nq, k, 2]
        (distance bits, global slot) over the global R best it holds."""
        from .exact import merge_candidates_device
        world, r = gathered.shape[0], gathered.shape[2]
        d, rows = merge_candidates_device(gathered, world, r, "dot_product")  # keys kept as they are
        dist, lrows = self.local.rerank_device(queries, k, _pairs(d, self._to_local(rows)))
        return _pairs(dist, self._to_global(lrows))

    @staticmethod
    def merge_final(gathered, k: int):
        """Phase 4 (root): gathered [world, nq, k, 2] -> (dist, global rows) [nq, k]."""
        from .exact import merge_candidates_device
        return merge_candidates_device(gathered, gathered.shape[0], k, "dot_product")

    def search_device(self, queries, k: int):
        """Every rank calls it; (dist, global rows) on the root, (None, None) elsewhere."""
        if self.world == 1:
            d, r = self.local.search_device(queries, k)
            return d, self._to_global(r)
        # The probe is split across the ranks (each probes a slice of the
        # batch against the replicated centroids) and exchanged.
        probes = self.probe_table(self.exchange(self.probe_slice(queries)), queries.shape[0])
        if self.peer is not None:
            return self._search_peer(queries, k, probes)
        mine = self.rerank_owned(queries, k, self.exchange(self.approx_candidates(queries, k, probes)))
        gathered = self.exchange(mine)
        if self.rank != 0:
            return None, None
        return self.merge_final(gathered, k)

    def _search_peer(self, queries, k, probes):
        import torch
        from . import _capi as capi
        nq = queries.shape[0]
        self.peer.ensure(nq, k)
        my_slot, bounds, blocks = self.peer.slots(nq)
        approx = self.approx_candidates(queries, k, probes, shared_bound=bounds)
        mine = self.rerank_owned(queries, k, self.exchange(approx)).contiguous()
        stream = torch.cuda.current_stream(queries.device).cuda_stream
        capi.check(capi.LIB.elips_b200_copy_device(self.local.device, my_slot, mine.data_ptr(), nq * k * 8, stream),
                   "elips_b200_copy_device")
        self.peer.finish_step(nq, stream)
        if self.rank != 0:
            return None, None
        out_dist = torch.empty((nq, k), dtype=torch.float32, device=queries.device)
        out_rows = torch.empty((nq, k), dtype=torch.int64, device=queries.device)
        capi.check(capi.LIB.elips_b200_merge_candidates_device(
            self.local.device, blocks, nq, self.world, k, METRICS_CODE["dot_product"], out_dist.data_ptr(),
            out_rows.data_ptr(), stream), "elips_b200_merge_candidates_device")
        return out_dist, out_rows
