"""Exact (brute-force) k-NN index on one B200.

Mirrors the reference's exhaustive index interface: ExactIndex
(include/elips/index_engine/ExactIndex.hpp:26-66; search at
src/ExactIndex.cpp:55-87) and GpuBruteForceIndex::search_batch
(src/gpu_engine/GpuBruteForceIndex.cpp:152-170). Rows are identified by their
insertion slot (0, 1, 2, ...); the caller keeps the slot -> RecordID map, as
GpuBruteForceIndex keeps `ids_`.

Distances follow src/Metrics.cpp:104-115 (cosine = 1 - dot on pre-normalised
vectors, euclidean = sqrt of the squared L2, dot_product = -dot); results are
ascending by (distance, slot).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np

from . import _capi as capi

METRICS = {"cosine": capi.METRIC_COSINE, "euclidean": capi.METRIC_EUCLIDEAN,
           "dot_product": capi.METRIC_DOT_PRODUCT}
PRECISIONS = {"fp32": capi.PRECISION_FP32, "fp16": capi.PRECISION_FP16,
              "int8": capi.PRECISION_INT8, "auto": capi.PRECISION_AUTO,
              "bf16": capi.PRECISION_BF16}


class DimensionMismatch(ValueError):
    """Raised where the reference throws elips::DimensionMismatch
    (src/ExactIndex.cpp:14-20)."""


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class ExactIndex:
    """Device-resident exhaustive index searched by the fused tensor-core kernel.

    precision: "fp32" (3xTF32, fp32-exact ranking), "fp16", "bf16", or "int8"
    (symmetric int8 codec: int8 rows and queries, dot_product only, exact int32
    scores).
    """

    def __init__(self, metric: str, dimension: int, precision: str = "fp32", device: int = 0):
        if metric not in METRICS:
            raise ValueError(f"unknown metric {metric!r}")
        if precision not in PRECISIONS:
            raise ValueError(f"unknown precision {precision!r}")
        self.metric = metric
        self.dimension = int(dimension)
        self.precision = precision
        self.device = int(device)
        self._in_dtype = np.int8 if precision == "int8" else np.float32
        handle = ctypes.c_void_p()
        capi.check(capi.LIB.elips_b200_exact_create(self.device, METRICS[metric], PRECISIONS[precision],
                                                    self.dimension, ctypes.byref(handle)),
                   "elips_b200_exact_create")
        self._h = handle

    # -- IndexPort ---------------------------------------------------------
    def add(self, rows: np.ndarray) -> None:
        """Appends rows (n x dimension) to the next slots."""
        rows = np.ascontiguousarray(rows, dtype=self._in_dtype)
        if rows.ndim != 2 or rows.shape[1] != self.dimension:
            raise DimensionMismatch("vector dimension does not match index")
        capi.check(capi.LIB.elips_b200_exact_add(self._h, _ptr(rows), rows.shape[0]),
                   "elips_b200_exact_add")

    def add_device(self, rows, stream=None) -> None:
        """Appends rows held in a CUDA tensor [n, dimension] (float32, int8 for int8)."""
        import torch
        if rows.dim() != 2 or rows.shape[1] != self.dimension:
            raise DimensionMismatch("vector dimension does not match index")
        rows = rows.contiguous()
        s = stream if stream is not None else torch.cuda.current_stream(rows.device).cuda_stream
        capi.check(capi.LIB.elips_b200_exact_add_device(self._h, rows.data_ptr(), rows.shape[0], s),
                   "elips_b200_exact_add_device")

    def insert(self, vector: np.ndarray) -> None:
        self.add(np.asarray(vector, dtype=self._in_dtype).reshape(1, -1))

    def size(self) -> int:
        """Rows ever added: the slot-number space results are reported in."""
        n = ctypes.c_size_t(0)
        capi.check(capi.LIB.elips_b200_exact_size(self._h, ctypes.byref(n)), "elips_b200_exact_size")
        return n.value

    def live(self) -> int:
        """Rows not removed."""
        n = ctypes.c_size_t(0)
        capi.check(capi.LIB.elips_b200_exact_live(self._h, ctypes.byref(n)), "elips_b200_exact_live")
        return n.value

    def remove(self, slot: int) -> bool:
        """Removes one row on the device (no rebuild); False if already removed."""
        r = ctypes.c_int(0)
        capi.check(capi.LIB.elips_b200_exact_remove(self._h, int(slot), ctypes.byref(r)), "elips_b200_exact_remove")
        return bool(r.value)

    def compact(self) -> np.ndarray:
        """Drops removed rows keeping order; returns each kept row's former slot."""
        out = np.empty(max(1, self.live()), np.uint32)
        capi.check(capi.LIB.elips_b200_exact_compact(self._h, _ptr(out), out.shape[0]), "elips_b200_exact_compact")
        return out[:self.live()]

    def export_snapshot(self) -> bytes:
        """The device rows (operands, norms, removal bits) as one blob."""
        n = ctypes.c_size_t(0)
        capi.check(capi.LIB.elips_b200_exact_snapshot_bytes(self._h, ctypes.byref(n)), "elips_b200_exact_snapshot_bytes")
        buf = np.empty(n.value, np.uint8)
        capi.check(capi.LIB.elips_b200_exact_export(self._h, _ptr(buf), buf.shape[0]), "elips_b200_exact_export")
        return buf.tobytes()

    def import_snapshot(self, blob: bytes) -> None:
        """Restores export_snapshot's blob into this (empty) index."""
        buf = np.frombuffer(blob, np.uint8)
        capi.check(capi.LIB.elips_b200_exact_import(self._h, _ptr(buf), buf.shape[0]), "elips_b200_exact_import")

    def search(self, query: np.ndarray, k: int) -> list[tuple[int, float]]:
        """IndexPort::search for one query: up to k (slot, distance) pairs."""
        d, r = self.search_batch(np.asarray(query).reshape(1, -1), k)
        return [(int(r[0, i]), float(d[0, i])) for i in range(d.shape[1]) if r[0, i] >= 0]

    def search_batch(self, queries: np.ndarray, k: int, mask: Optional[np.ndarray] = None,
                     out_dist: Optional[np.ndarray] = None,
                     out_rows: Optional[np.ndarray] = None) -> tuple[np.ndarray, np.ndarray]:
        """Host arrays in, host arrays out: (distances [nq, k] fp32, slots [nq, k] int64).
        Unfilled slots hold (+inf, -1). mask: uint32 words, bit i = slot i eligible.
        out_dist / out_rows: optional preallocated (e.g. pinned) C-contiguous outputs."""
        q = np.ascontiguousarray(queries, dtype=self._in_dtype)
        if q.ndim != 2 or q.shape[1] != self.dimension:
            raise DimensionMismatch("query dimension does not match index")
        nq = q.shape[0]
        dist = np.empty((nq, k), dtype=np.float32) if out_dist is None else out_dist
        rows = np.empty((nq, k), dtype=np.int64) if out_rows is None else out_rows
        if dist.shape != (nq, k) or rows.shape != (nq, k) or dist.dtype != np.float32 \
                or rows.dtype != np.int64 or not dist.flags.c_contiguous or not rows.flags.c_contiguous:
            raise ValueError("outputs must be C-contiguous float32 / int64 arrays of shape (nq, k)")
        m = None
        if mask is not None:
            m = np.ascontiguousarray(mask, dtype=np.uint32)
            if m.size < (self.size() + 31) // 32:
                raise ValueError("mask has fewer words than ceil(size / 32)")
        capi.check(capi.LIB.elips_b200_exact_search(self._h, _ptr(q), nq, k,
                                                    _ptr(m) if m is not None else None,
                                                    _ptr(dist), _ptr(rows)),
                   "elips_b200_exact_search")
        return dist, rows

    # -- device-pointer entry points (torch tensors as plumbing) -----------
    def search_device(self, queries, k: int, mask=None, out_dist=None, out_rows=None, stream=None):
        """queries: CUDA tensor [nq, dimension] (float32, int8 for int8). Asynchronous on
        `stream` (default: torch's current stream). Returns (dist, rows) CUDA tensors."""
        import torch
        nq = queries.shape[0]
        if queries.shape[1] != self.dimension:
            raise DimensionMismatch("query dimension does not match index")
        if out_dist is None:
            out_dist = torch.empty((nq, k), dtype=torch.float32, device=queries.device)
        if out_rows is None:
            out_rows = torch.empty((nq, k), dtype=torch.int64, device=queries.device)
        s = stream if stream is not None else torch.cuda.current_stream(queries.device).cuda_stream
        capi.check(capi.LIB.elips_b200_exact_search_device(
            self._h, queries.data_ptr(), nq, k, mask.data_ptr() if mask is not None else None,
            out_dist.data_ptr(), out_rows.data_ptr(), s), "elips_b200_exact_search_device")
        return out_dist, out_rows

    def search_candidates_device(self, queries, k: int, row_offset: int, out_cand, mask=None, stream=None):
        """Shard-level search: writes [nq, k, 2] uint32-as-int32 candidate pairs to out_cand."""
        import torch
        s = stream if stream is not None else torch.cuda.current_stream(queries.device).cuda_stream
        capi.check(capi.LIB.elips_b200_exact_search_candidates_device(
            self._h, queries.data_ptr(), queries.shape[0], k,
            mask.data_ptr() if mask is not None else None, row_offset, out_cand.data_ptr(), s),
            "elips_b200_exact_search_candidates_device")
        return out_cand

    def search_candidates_shared_device(self, queries, k: int, row_offset: int, out_cand, shared_bound, mask=None,
                                        stream=None):
        """Shard-level search whose per-query admission bounds (shared_bound:
        an int32 CUDA tensor [nq] of ordered keys, all ones = none) are shared
        with the other shards searching the same queries."""
        import torch
        s = stream if stream is not None else torch.cuda.current_stream(queries.device).cuda_stream
        capi.check(capi.LIB.elips_b200_exact_search_candidates_shared_device(
            self._h, queries.data_ptr(), queries.shape[0], k, mask.data_ptr() if mask is not None else None,
            row_offset, out_cand.data_ptr(), shared_bound.data_ptr(), s),
            "elips_b200_exact_search_candidates_shared_device")
        return out_cand

    def close(self) -> None:
        if getattr(self, "_h", None):
            capi.LIB.elips_b200_exact_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def merge_candidates_device(cand, lists: int, k: int, metric: str, out_dist=None, out_rows=None,
                            stream=None):
    """Final top-k over `lists` blocks of [nq, k] candidate pairs (block-major)."""
    import torch
    nq = cand.numel() // (2 * lists * k) if lists else 0
    dev = cand.device
    if out_dist is None:
        out_dist = torch.empty((nq, k), dtype=torch.float32, device=dev)
    if out_rows is None:
        out_rows = torch.empty((nq, k), dtype=torch.int64, device=dev)
    s = stream if stream is not None else torch.cuda.current_stream(dev).cuda_stream
    capi.check(capi.LIB.elips_b200_merge_candidates_device(
        dev.index, cand.data_ptr(), nq, lists, k, METRICS[metric], out_dist.data_ptr(),
        out_rows.data_ptr(), s), "elips_b200_merge_candidates_device")
    return out_dist, out_rows


class DynamicBatcher:
    """Coalesces concurrent single-query searches on an ExactIndex into batched
    launches (elips::gpu::DynamicBatcher, src/gpu_engine/DynamicBatcher.cpp).
    search() blocks until the caller's batch ran; safe to call from many
    threads (the GIL is released inside the C call)."""

    def __init__(self, index: ExactIndex, window_us: int = 500, max_batch: int = 256):
        self.index = index
        h = ctypes.c_void_p()
        capi.check(capi.LIB.elips_b200_batcher_create(index._h, int(window_us), int(max_batch), ctypes.byref(h)),
                   "elips_b200_batcher_create")
        self._h = h

    def search(self, query: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
        q = np.ascontiguousarray(query, dtype=self.index._in_dtype).reshape(-1)
        if q.shape[0] != self.index.dimension:
            raise DimensionMismatch("query dimension does not match index")
        dist = np.empty(k, np.float32)
        rows = np.empty(k, np.int64)
        capi.check(capi.LIB.elips_b200_batcher_search(self._h, _ptr(q), k, _ptr(dist), _ptr(rows)),
                   "elips_b200_batcher_search")
        return dist, rows

    def flush(self) -> None:
        """DynamicBatcher::flush: serve the pending queries now, without
        waiting for the window; returns when they have been served."""
        capi.check(capi.LIB.elips_b200_batcher_flush(self._h), "elips_b200_batcher_flush")

    def pending(self) -> int:
        """Queries queued and not yet taken into a batch."""
        n = ctypes.c_uint64(0)
        capi.check(capi.LIB.elips_b200_batcher_pending(self._h, ctypes.byref(n)), "elips_b200_batcher_pending")
        return n.value

    def stats(self) -> dict:
        l, q = ctypes.c_uint64(0), ctypes.c_uint64(0)
        capi.check(capi.LIB.elips_b200_batcher_stats(self._h, ctypes.byref(l), ctypes.byref(q)),
                   "elips_b200_batcher_stats")
        return {"kernel_launches": l.value, "queries_coalesced": q.value,
                "avg_batch_size": q.value / l.value if l.value else 0.0}

    def close(self) -> None:
        if getattr(self, "_h", None):
            capi.LIB.elips_b200_batcher_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
