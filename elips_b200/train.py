"""Index build on one B200, bit-identical to the reference's trainers.

* kmeans              quant::detail::kmeans (src/quant_engine/KMeans.cpp:182-247)
* train_pq_codebook   quant::detail::train_pq_codebook (KMeans.cpp:249-268)
* ivf_assign          IvfIndexState::assign_vectors_to_centroids
                      (src/gpu_engine/detail/IvfIndexState.cpp:167-191)
* ivf_train           IvfIndexState::rebuild_from_current_data: train_centroids
                      then the final assignment (IvfIndexState.cpp:118-208)
* ivfpq_train         GpuIVFPQIndex's model build: ivf_train, then the residual
                      PQ codebook (10 rounds) and codes (GpuIVFPQIndex.cpp:88-131)

numpy in, numpy out; the *_device variants take and return torch CUDA tensors
and run on the tensor's device and current stream.
"""
from __future__ import annotations

import numpy as np

from . import _capi as capi
from .exact import METRICS


def _rows(rows) -> np.ndarray:
    x = np.ascontiguousarray(rows, np.float32)
    if x.ndim != 2:
        raise ValueError("rows must be [n, dimension]")
    return x


def target_lists(requested: int, n: int) -> int:
    """normalize_target_lists (IvfIndexState.cpp:15-18): max(1, min(requested, n))."""
    return max(1, min(int(requested), int(n)))


def kmeans(rows, k: int, iters: int, device: int = 0) -> np.ndarray:
    x = _rows(rows)
    out = np.empty((k, x.shape[1]), np.float32)
    capi.check(capi.LIB.elips_b200_kmeans(device, x.ctypes.data, x.shape[0], x.shape[1], k, iters,
                                          out.ctypes.data, 0, None), "elips_b200_kmeans")
    return out


def train_pq_codebook(rows, pq_dim: int, ksub: int, iters: int = 10, device: int = 0) -> np.ndarray:
    """Codebook [pq_dim][ksub][dimension / pq_dim]."""
    x = _rows(rows)
    n, d = x.shape
    out = np.empty((pq_dim, ksub, d // pq_dim), np.float32)
    capi.check(capi.LIB.elips_b200_train_pq_codebook(device, x.ctypes.data, n, d, pq_dim, ksub, iters,
                                                     out.ctypes.data, 0, None), "elips_b200_train_pq_codebook")
    return out


def ivf_nearest(metric: str, rows, centroids, device: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """(nearest list [n] uint32, its distance [n] float32) for every row."""
    x, c = _rows(rows), _rows(centroids)
    out = np.empty(x.shape[0], np.uint32)
    dist = np.empty(x.shape[0], np.float32)
    capi.check(capi.LIB.elips_b200_ivf_assign(device, METRICS[metric], x.ctypes.data, x.shape[0], x.shape[1],
                                              c.ctypes.data, c.shape[0], out.ctypes.data, dist.ctypes.data, 0,
                                              None), "elips_b200_ivf_assign")
    return out, dist


def ivf_assign(metric: str, rows, centroids, device: int = 0) -> np.ndarray:
    x, c = _rows(rows), _rows(centroids)
    out = np.empty(x.shape[0], np.uint32)
    capi.check(capi.LIB.elips_b200_ivf_assign(device, METRICS[metric], x.ctypes.data, x.shape[0], x.shape[1],
                                              c.ctypes.data, c.shape[0], out.ctypes.data, None, 0, None),
               "elips_b200_ivf_assign")
    return out


def ivf_train(metric: str, rows, n_lists: int, iters: int, device: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """(centroids [lists][d], assignments [n]) with lists = target_lists(n_lists, n)."""
    x = _rows(rows)
    n, d = x.shape
    lists = target_lists(n_lists, n)
    cent = np.empty((lists, d), np.float32)
    asg = np.empty(n, np.uint32)
    capi.check(capi.LIB.elips_b200_ivf_train(device, METRICS[metric], x.ctypes.data, n, d, lists, iters,
                                             cent.ctypes.data, asg.ctypes.data, 0, None), "elips_b200_ivf_train")
    return cent, asg


def ivfpq_train(metric: str, rows, n_lists: int, iters: int, pq_dim: int, pq_bits: int = 8, device: int = 0):
    """(centroids, assignments, codebook [pq_dim][2^pq_bits][d/pq_dim], codes [n][pq_dim])."""
    x = _rows(rows)
    n, d = x.shape
    lists = target_lists(n_lists, n)
    cent = np.empty((lists, d), np.float32)
    asg = np.empty(n, np.uint32)
    cb = np.empty((pq_dim, 1 << pq_bits, d // pq_dim), np.float32)
    codes = np.empty((n, pq_dim), np.uint8)
    capi.check(capi.LIB.elips_b200_ivfpq_train(device, METRICS[metric], x.ctypes.data, n, d, lists, iters, pq_dim,
                                               pq_bits, cent.ctypes.data, asg.ctypes.data, cb.ctypes.data,
                                               codes.ctypes.data, 0, None), "elips_b200_ivfpq_train")
    return cent, asg, cb, codes


def _stream(t):
    import torch
    return torch.cuda.current_stream(t.device).cuda_stream


def ivf_train_device(metric: str, rows, n_lists: int, iters: int):
    """ivf_train on a CUDA float32 tensor [n, d]: (centroids, assignments int32)."""
    import torch
    x = rows.contiguous()
    n, d = x.shape
    lists = target_lists(n_lists, n)
    cent = torch.empty((lists, d), dtype=torch.float32, device=x.device)
    asg = torch.empty(n, dtype=torch.int32, device=x.device)
    capi.check(capi.LIB.elips_b200_ivf_train(x.device.index, METRICS[metric], x.data_ptr(), n, d, lists, iters,
                                             cent.data_ptr(), asg.data_ptr(), 1, _stream(x)), "elips_b200_ivf_train")
    return cent, asg


def ivfpq_train_device(metric: str, rows, n_lists: int, iters: int, pq_dim: int, pq_bits: int = 8,
                       with_codes: bool = True):
    """ivfpq_train on a CUDA float32 tensor: (centroids, assignments int32,
    codebook, codes uint8 or None)."""
    import torch
    x = rows.contiguous()
    n, d = x.shape
    lists = target_lists(n_lists, n)
    cent = torch.empty((lists, d), dtype=torch.float32, device=x.device)
    asg = torch.empty(n, dtype=torch.int32, device=x.device)
    cb = torch.empty((pq_dim, 1 << pq_bits, d // pq_dim), dtype=torch.float32, device=x.device)
    codes = torch.empty((n, pq_dim), dtype=torch.uint8, device=x.device) if with_codes else None
    capi.check(capi.LIB.elips_b200_ivfpq_train(x.device.index, METRICS[metric], x.data_ptr(), n, d, lists, iters,
                                               pq_dim, pq_bits, cent.data_ptr(), asg.data_ptr(), cb.data_ptr(),
                                               codes.data_ptr() if codes is not None else None, 1, _stream(x)),
               "elips_b200_ivfpq_train")
    return cent, asg, cb, codes
