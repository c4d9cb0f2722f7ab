"""Quantized exhaustive search and the GpuPort primitives on one B200.

QuantizedIndex mirrors ExactIndex with a trained Quantizer attached
(include/elips/index_engine/ExactIndex.hpp:26-66, compressed search at
src/ExactIndex.cpp:62-71): rows are stored as codes on the device and every
query is scored with the codec's lookup table, bit for bit as
ProductQuantizer::make_lut / lut_distance (src/quant_engine/
ProductQuantizer.cpp:118-183) and ScalarQuantizer::make_lut / lut_distance
(src/quant_engine/ScalarQuantizer.cpp:83-128).

compute_distances_batch / top_k mirror GpuPort's primitives
(include/elips/gpu_engine/GpuPort.hpp:65-82).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np

from . import _capi as capi
from .exact import METRICS, DimensionMismatch

CODECS = {"pq": capi.CODEC_PQ, "opq": capi.CODEC_OPQ, "sq8": capi.CODEC_SQ8}


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class QuantizedIndex:
    """codec "pq"/"opq": codebook [pq_dim][2^pq_bits][dimension/pq_dim] (and an
    orthonormal rotation [dimension][dimension] for "opq"); codec "sq8": mins
    and scales [dimension] each (ScalarQuantizer)."""

    def __init__(self, codec: str, metric: str, dimension: int, *, codebook=None, rotation=None,
                 mins=None, scales=None, pq_bits: int = 8, device: int = 0):
        if codec not in CODECS:
            raise ValueError(f"unknown codec {codec!r}")
        self.codec, self.metric, self.dimension, self.device = codec, metric, int(dimension), int(device)
        rot = None
        if codec == "sq8":
            params = np.ascontiguousarray(np.concatenate([np.asarray(mins, np.float32),
                                                          np.asarray(scales, np.float32)]))
            pq_dim, self.code_bytes = 0, self.dimension
        else:
            params = np.ascontiguousarray(codebook, dtype=np.float32)
            pq_dim = params.shape[0]
            self.code_bytes = pq_dim
            if rotation is not None:
                rot = np.ascontiguousarray(rotation, dtype=np.float32)
        self._keep = (params, rot)
        h = ctypes.c_void_p()
        capi.check(capi.LIB.elips_b200_quant_create(self.device, CODECS[codec], METRICS[metric], self.dimension,
                                                    pq_dim, pq_bits, _ptr(params),
                                                    _ptr(rot) if rot is not None else None, ctypes.byref(h)),
                   "elips_b200_quant_create")
        self._h = h

    def add(self, rows: np.ndarray) -> None:
        """IndexPort::insert for fp32 rows, encoded on the device by the codec."""
        rows = np.ascontiguousarray(rows, dtype=np.float32)
        if rows.ndim != 2 or rows.shape[1] != self.dimension:
            raise DimensionMismatch("vector dimension does not match index")
        capi.check(capi.LIB.elips_b200_quant_add(self._h, _ptr(rows), rows.shape[0]), "elips_b200_quant_add")

    def add_codes(self, codes: np.ndarray) -> None:
        codes = np.ascontiguousarray(codes, dtype=np.uint8)
        if codes.ndim != 2 or codes.shape[1] != self.code_bytes:
            raise ValueError("codes must be n x code_bytes")
        capi.check(capi.LIB.elips_b200_quant_add_codes(self._h, _ptr(codes), codes.shape[0]),
                   "elips_b200_quant_add_codes")

    def size(self) -> int:
        n = ctypes.c_size_t(0)
        capi.check(capi.LIB.elips_b200_quant_size(self._h, ctypes.byref(n)), "elips_b200_quant_size")
        return n.value

    def search_batch(self, queries: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
        q = np.ascontiguousarray(queries, dtype=np.float32)
        if q.ndim != 2 or q.shape[1] != self.dimension:
            raise DimensionMismatch("query dimension does not match index")
        nq = q.shape[0]
        dist = np.empty((nq, k), np.float32)
        rows = np.empty((nq, k), np.int64)
        capi.check(capi.LIB.elips_b200_quant_search(self._h, _ptr(q), nq, k, _ptr(dist), _ptr(rows)),
                   "elips_b200_quant_search")
        return dist, rows

    def search_device(self, queries, k: int, stream=None):
        import torch
        nq = queries.shape[0]
        d = torch.empty((nq, k), dtype=torch.float32, device=queries.device)
        r = torch.empty((nq, k), dtype=torch.int64, device=queries.device)
        s = stream if stream is not None else torch.cuda.current_stream(queries.device).cuda_stream
        capi.check(capi.LIB.elips_b200_quant_search_device(self._h, queries.data_ptr(), nq, k, d.data_ptr(),
                                                           r.data_ptr(), s), "elips_b200_quant_search_device")
        return d, r

    def close(self) -> None:
        if getattr(self, "_h", None):
            capi.LIB.elips_b200_quant_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def compute_distances_batch(queries: np.ndarray, database: np.ndarray, metric: str,
                            device: int = 0) -> np.ndarray:
    """GpuPort::compute_distances_batch over host arrays: [nq, nb] distances,
    bit for bit elips::distance."""
    q = np.ascontiguousarray(queries, np.float32)
    db = np.ascontiguousarray(database, np.float32)
    if q.shape[1] != db.shape[1]:
        raise DimensionMismatch("query and database dimensions differ")
    out = np.empty((q.shape[0], db.shape[0]), np.float32)
    capi.check(capi.LIB.elips_b200_compute_distances_batch(device, _ptr(q), _ptr(db), _ptr(out), q.shape[0],
                                                           db.shape[0], q.shape[1], METRICS[metric], 0, None),
               "elips_b200_compute_distances_batch")
    return out


def top_k(distances: np.ndarray, k: int, device: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """GpuPort::top_k over a host [nq, nb] matrix: (indices uint32, values fp32), [nq, k]."""
    d = np.ascontiguousarray(distances, np.float32)
    nq, nb = d.shape
    idx = np.empty((nq, k), np.uint32)
    val = np.empty((nq, k), np.float32)
    capi.check(capi.LIB.elips_b200_top_k(device, _ptr(d), _ptr(idx), _ptr(val), nq, nb, k, 0, None),
               "elips_b200_top_k")
    return idx, val


def normalize_rows(rows: np.ndarray, device: int = 0) -> np.ndarray:
    """Vector::normalized of every row (Vector.hpp:25-44), on the device."""
    x = np.ascontiguousarray(rows, np.float32)
    out = np.empty_like(x)
    n, d = x.shape
    capi.check(capi.LIB.elips_b200_normalize_rows(device, x.ctypes.data, out.ctypes.data, n, d, 0, None),
               "elips_b200_normalize_rows")
    return out
