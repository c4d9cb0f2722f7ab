"""IVF indexes on one B200: GpuIVFPQIndex (src/gpu_engine/GpuIVFPQIndex.cpp)
and GpuIVFFlatIndex (src/gpu_engine/GpuIVFFlatIndex.cpp), with their trained
model imported as import_snapshot does (GpuIVFPQIndex.cpp:327-348).

Search follows GpuIVFPQIndex::search (:161-237): exact probe of the nprobe
nearest lists, approximate scoring of their members from the residual codes,
exact rerank of the best R = max(4k, k) on the raw vectors. Returned
distances are the exact ones, ascending by (distance, slot).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np

from . import _capi as capi
from .exact import METRICS, DimensionMismatch


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class IvfPqIndex:
    def __init__(self, metric: str, dimension: int, centroids: np.ndarray, codebook: np.ndarray,
                 nprobe: int, pq_bits: int = 8, device: int = 0):
        self.metric, self.dimension, self.device = metric, int(dimension), int(device)
        cent = np.ascontiguousarray(centroids, np.float32)
        cb = np.ascontiguousarray(codebook, np.float32)
        if cent.shape[1] != self.dimension:
            raise DimensionMismatch("centroid dimension does not match index")
        self.n_lists, self.pq_dim, self.pq_bits = cent.shape[0], cb.shape[0], int(pq_bits)
        self.nprobe = max(1, int(nprobe))
        h = ctypes.c_void_p()
        capi.check(capi.LIB.elips_b200_ivfpq_create(self.device, METRICS[metric], self.dimension, self.n_lists,
                                                    int(nprobe), self.pq_dim, int(pq_bits), _ptr(cent), _ptr(cb),
                                                    ctypes.byref(h)), "elips_b200_ivfpq_create")
        self._h = h

    def add(self, vectors: np.ndarray, assignments: np.ndarray, codes: Optional[np.ndarray] = None) -> None:
        """Host rows, their list ids, and optionally their residual codes."""
        v = np.ascontiguousarray(vectors, np.float32)
        a = np.ascontiguousarray(assignments, np.uint32)
        if v.ndim != 2 or v.shape[1] != self.dimension:
            raise DimensionMismatch("vector dimension does not match index")
        c = None if codes is None else np.ascontiguousarray(codes, np.uint8)
        capi.check(capi.LIB.elips_b200_ivfpq_add(self._h, _ptr(v), _ptr(a), _ptr(c) if c is not None else None,
                                                 v.shape[0]), "elips_b200_ivfpq_add")

    def add_device(self, vectors, assignments, codes=None, stream=None) -> None:
        """CUDA tensors: vectors [n, d] float32, assignments [n] int32 (list ids)."""
        import torch
        if vectors.shape[1] != self.dimension:
            raise DimensionMismatch("vector dimension does not match index")
        vectors, assignments = vectors.contiguous(), assignments.contiguous()
        s = stream if stream is not None else torch.cuda.current_stream(vectors.device).cuda_stream
        capi.check(capi.LIB.elips_b200_ivfpq_add_device(self._h, vectors.data_ptr(), assignments.data_ptr(),
                                                        codes.data_ptr() if codes is not None else None,
                                                        vectors.shape[0], s), "elips_b200_ivfpq_add_device")

    def remove(self, slot: int) -> None:
        """IvfIndexState::remove: the last slot's row moves into `slot`."""
        capi.check(capi.LIB.elips_b200_ivfpq_remove(self._h, int(slot)), "elips_b200_ivfpq_remove")

    def rebuild_codes(self) -> None:
        """GpuIVFPQIndex::rebuild_codes: retrain the codebook on all residuals, re-encode."""
        capi.check(capi.LIB.elips_b200_ivfpq_rebuild_codes(self._h), "elips_b200_ivfpq_rebuild_codes")

    def export_snapshot(self) -> dict:
        """IndexSnapshot's fields in slot order: centroids, assignments,
        vectors, codebook, codes (elips_b200_ivfpq_create + add rebuild it)."""
        n, d = self.size(), self.dimension
        out = {"centroids": np.empty((self.n_lists, d), np.float32), "assignments": np.empty(n, np.uint32),
               "vectors": np.empty((n, d), np.float32),
               "codebook": np.empty((self.pq_dim, 1 << self.pq_bits, d // self.pq_dim), np.float32),
               "codes": np.empty((n, self.pq_dim), np.uint8)}
        capi.check(capi.LIB.elips_b200_ivfpq_export(self._h, _ptr(out["centroids"]), _ptr(out["assignments"]),
                                                    _ptr(out["vectors"]), _ptr(out["codebook"]), _ptr(out["codes"])),
                   "elips_b200_ivfpq_export")
        return out

    def size(self) -> int:
        n = ctypes.c_size_t(0)
        capi.check(capi.LIB.elips_b200_ivfpq_size(self._h, ctypes.byref(n)), "elips_b200_ivfpq_size")
        return n.value

    def set_nprobe(self, nprobe: int) -> None:
        capi.check(capi.LIB.elips_b200_ivfpq_set_nprobe(self._h, int(nprobe)), "elips_b200_ivfpq_set_nprobe")
        self.nprobe = max(1, int(nprobe))

    def set_list_range(self, lo: int, hi: int) -> None:
        """Own only lists [lo, hi) (one GPU's share of a list-sharded index)."""
        capi.check(capi.LIB.elips_b200_ivfpq_set_list_range(self._h, int(lo), int(hi)),
                   "elips_b200_ivfpq_set_list_range")

    def set_owned_lists(self, owned) -> None:
        """Own only the lists where `owned` (bool array [n_lists]) is true."""
        owned = np.asarray(owned, bool)
        words = np.zeros((self.n_lists + 31) // 32, np.uint32)
        idx = np.nonzero(owned)[0]
        np.bitwise_or.at(words, idx >> 5, (np.uint32(1) << (idx & 31).astype(np.uint32)))
        capi.check(capi.LIB.elips_b200_ivfpq_set_owned_lists(self._h, _ptr(words), words.size),
                   "elips_b200_ivfpq_set_owned_lists")

    def probe_device(self, queries, stream=None):
        """The nprobe nearest lists of each query: [nq, nprobe] int32, ascending."""
        import torch
        nq = queries.shape[0]
        nprobe = min(self.nprobe, self.n_lists)
        out = torch.empty((nq, nprobe), dtype=torch.int32, device=queries.device)
        s = stream if stream is not None else torch.cuda.current_stream(queries.device).cuda_stream
        capi.check(capi.LIB.elips_b200_ivfpq_probe_device(self._h, queries.data_ptr(), nq, out.data_ptr(), s),
                   "elips_b200_ivfpq_probe_device")
        return out

    def search_candidates_device(self, queries, k: int, out=None, stream=None, probes=None, shared_bound=None):
        """The approximate stage: [nq, 4k, 2] int32 (distance bits, slot),
        ascending; `probes` ([nq, nprobe] int32 CUDA tensor, probe_device's
        output) skips the probe. `shared_bound` (device address of nq uint32
        admission bounds, possibly a peer GPU's, shared by the shards of one
        list-sharded index searching this batch) replaces the search's own."""
        import torch
        nq = queries.shape[0]
        if out is None:
            out = torch.empty((nq, 4 * k, 2), dtype=torch.int32, device=queries.device)
        s = stream if stream is not None else torch.cuda.current_stream(queries.device).cuda_stream
        if shared_bound is not None:
            if probes is not None:
                probes = probes.contiguous()
            capi.check(capi.LIB.elips_b200_ivfpq_search_candidates_shared_device(
                self._h, queries.data_ptr(), nq, k, None if probes is None else probes.data_ptr(), out.data_ptr(),
                shared_bound, s), "elips_b200_ivfpq_search_candidates_shared_device")
        elif probes is None:
            capi.check(capi.LIB.elips_b200_ivfpq_search_candidates_device(self._h, queries.data_ptr(), nq, k,
                                                                          out.data_ptr(), s),
                       "elips_b200_ivfpq_search_candidates_device")
        else:
            probes = probes.contiguous()
            capi.check(capi.LIB.elips_b200_ivfpq_search_candidates_probed_device(
                self._h, queries.data_ptr(), nq, k, probes.data_ptr(), out.data_ptr(), s),
                "elips_b200_ivfpq_search_candidates_probed_device")
        return out

    def rerank_device(self, queries, k: int, cand, out_dist=None, out_rows=None, stream=None):
        """The exact stage over cand [nq, 4k, 2] (slot -1 = none): (dist, slot) [nq, k]."""
        import torch
        nq = queries.shape[0]
        if out_dist is None:
            out_dist = torch.empty((nq, k), dtype=torch.float32, device=queries.device)
            out_rows = torch.empty((nq, k), dtype=torch.int64, device=queries.device)
        cand = cand.contiguous()
        s = stream if stream is not None else torch.cuda.current_stream(queries.device).cuda_stream
        capi.check(capi.LIB.elips_b200_ivfpq_rerank_device(self._h, queries.data_ptr(), nq, k, cand.data_ptr(),
                                                           out_dist.data_ptr(), out_rows.data_ptr(), s),
                   "elips_b200_ivfpq_rerank_device")
        return out_dist, out_rows

    def codes(self) -> np.ndarray:
        """Residual codes of every row in slot order (export_snapshot's pq.codes)."""
        import torch
        out = torch.empty((max(self.size(), 1), self.pq_dim), dtype=torch.uint8, device=f"cuda:{self.device}")
        capi.check(capi.LIB.elips_b200_ivfpq_codes_device(self._h, out.data_ptr(),
                                                          torch.cuda.current_stream(out.device).cuda_stream),
                   "elips_b200_ivfpq_codes_device")
        torch.cuda.synchronize(out.device)
        return out[:self.size()].cpu().numpy()

    def search_batch(self, queries: np.ndarray, k: int, out_dist=None, out_rows=None):
        q = np.ascontiguousarray(queries, np.float32)
        if q.ndim != 2 or q.shape[1] != self.dimension:
            raise DimensionMismatch("query dimension does not match index")
        nq = q.shape[0]
        dist = np.empty((nq, k), np.float32) if out_dist is None else out_dist
        rows = np.empty((nq, k), np.int64) if out_rows is None else out_rows
        capi.check(capi.LIB.elips_b200_ivfpq_search(self._h, _ptr(q), nq, k, _ptr(dist), _ptr(rows)),
                   "elips_b200_ivfpq_search")
        return dist, rows

    def search_device(self, queries, k: int, out_dist=None, out_rows=None, stream=None):
        import torch
        nq = queries.shape[0]
        if out_dist is None:
            out_dist = torch.empty((nq, k), dtype=torch.float32, device=queries.device)
            out_rows = torch.empty((nq, k), dtype=torch.int64, device=queries.device)
        s = stream if stream is not None else torch.cuda.current_stream(queries.device).cuda_stream
        capi.check(capi.LIB.elips_b200_ivfpq_search_device(self._h, queries.data_ptr(), nq, k, out_dist.data_ptr(),
                                                           out_rows.data_ptr(), s), "elips_b200_ivfpq_search_device")
        return out_dist, out_rows

    def close(self) -> None:
        if getattr(self, "_h", None):
            capi.LIB.elips_b200_ivfpq_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class IvfFlatIndex:
    """GpuIVFFlatIndex: probe the nprobe nearest lists, rank their members
    exactly (GpuIVFFlatIndex.cpp:44-103). Results ascend by (distance, gather
    position): the probed lists' members in probe order, then member order."""

    def __init__(self, metric: str, dimension: int, centroids: np.ndarray, nprobe: int, device: int = 0):
        self.metric, self.dimension, self.device = metric, int(dimension), int(device)
        cent = np.ascontiguousarray(centroids, np.float32)
        if cent.shape[1] != self.dimension:
            raise DimensionMismatch("centroid dimension does not match index")
        self.n_lists = cent.shape[0]
        h = ctypes.c_void_p()
        capi.check(capi.LIB.elips_b200_ivfflat_create(self.device, METRICS[metric], self.dimension, self.n_lists,
                                                      int(nprobe), _ptr(cent), ctypes.byref(h)),
                   "elips_b200_ivfflat_create")
        self._h = h

    def add(self, vectors: np.ndarray, assignments: np.ndarray) -> None:
        v = np.ascontiguousarray(vectors, np.float32)
        a = np.ascontiguousarray(assignments, np.uint32)
        if v.ndim != 2 or v.shape[1] != self.dimension:
            raise DimensionMismatch("vector dimension does not match index")
        capi.check(capi.LIB.elips_b200_ivfflat_add(self._h, _ptr(v), _ptr(a), v.shape[0]), "elips_b200_ivfflat_add")

    def add_device(self, vectors, assignments, stream=None) -> None:
        """CUDA tensors: vectors [n, d] float32, assignments [n] int32 (list ids)."""
        import torch
        if vectors.shape[1] != self.dimension:
            raise DimensionMismatch("vector dimension does not match index")
        vectors, assignments = vectors.contiguous(), assignments.contiguous()
        s = stream if stream is not None else torch.cuda.current_stream(vectors.device).cuda_stream
        capi.check(capi.LIB.elips_b200_ivfflat_add_device(self._h, vectors.data_ptr(), assignments.data_ptr(),
                                                          vectors.shape[0], s), "elips_b200_ivfflat_add_device")

    def remove(self, slot: int) -> None:
        """IvfIndexState::remove: the last slot's row moves into `slot`."""
        capi.check(capi.LIB.elips_b200_ivfflat_remove(self._h, int(slot)), "elips_b200_ivfflat_remove")

    def export_snapshot(self) -> dict:
        """centroids, assignments and vectors in slot order."""
        n, d = self.size(), self.dimension
        out = {"centroids": np.empty((self.n_lists, d), np.float32), "assignments": np.empty(n, np.uint32),
               "vectors": np.empty((n, d), np.float32)}
        capi.check(capi.LIB.elips_b200_ivfflat_export(self._h, _ptr(out["centroids"]), _ptr(out["assignments"]),
                                                      _ptr(out["vectors"])), "elips_b200_ivfflat_export")
        return out

    def size(self) -> int:
        n = ctypes.c_size_t(0)
        capi.check(capi.LIB.elips_b200_ivfflat_size(self._h, ctypes.byref(n)), "elips_b200_ivfflat_size")
        return n.value

    def set_nprobe(self, nprobe: int) -> None:
        capi.check(capi.LIB.elips_b200_ivfflat_set_nprobe(self._h, int(nprobe)), "elips_b200_ivfflat_set_nprobe")

    def search_batch(self, queries: np.ndarray, k: int, out_dist=None, out_rows=None):
        q = np.ascontiguousarray(queries, np.float32)
        if q.ndim != 2 or q.shape[1] != self.dimension:
            raise DimensionMismatch("query dimension does not match index")
        nq = q.shape[0]
        dist = np.empty((nq, k), np.float32) if out_dist is None else out_dist
        rows = np.empty((nq, k), np.int64) if out_rows is None else out_rows
        capi.check(capi.LIB.elips_b200_ivfflat_search(self._h, _ptr(q), nq, k, _ptr(dist), _ptr(rows)),
                   "elips_b200_ivfflat_search")
        return dist, rows

    def search_device(self, queries, k: int, out_dist=None, out_rows=None, stream=None):
        import torch
        nq = queries.shape[0]
        if out_dist is None:
            out_dist = torch.empty((nq, k), dtype=torch.float32, device=queries.device)
            out_rows = torch.empty((nq, k), dtype=torch.int64, device=queries.device)
        s = stream if stream is not None else torch.cuda.current_stream(queries.device).cuda_stream
        capi.check(capi.LIB.elips_b200_ivfflat_search_device(self._h, queries.data_ptr(), nq, k, out_dist.data_ptr(),
                                                             out_rows.data_ptr(), s),
                   "elips_b200_ivfflat_search_device")
        return out_dist, out_rows

    def close(self) -> None:
        if getattr(self, "_h", None):
            capi.LIB.elips_b200_ivfflat_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
