"""ctypes binding of include/elips_b200.h.

Loads the in-tree libelips_b200.so. There is no fallback: if the library is
missing or fails to load, importing this module raises.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int, c_int64, c_size_t, c_uint32, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libelips_b200.so"

OK = 0
DEVICE_NOT_FOUND = 1
INSUFFICIENT_MEMORY = 2
KERNEL_LAUNCH_FAILED = 3
TRANSFER_FAILED = 4
INDEX_BUILD_FAILED = 5
UNSUPPORTED_METRIC = 6
INITIALIZATION_FAILED = 7
BACKEND_UNAVAILABLE = 8
DIMENSION_MISMATCH = 9
INVALID_ARGUMENT = 10
DEVICE_TIMEOUT = 11

METRIC_COSINE = 0
METRIC_EUCLIDEAN = 1
METRIC_DOT_PRODUCT = 2

PRECISION_FP32 = 0
PRECISION_FP16 = 1
PRECISION_INT8 = 2
PRECISION_AUTO = 3
PRECISION_BF16 = 4

CODEC_PQ = 1
CODEC_OPQ = 2
CODEC_SQ8 = 3

# (name, restype, argtypes) for every entry point in include/elips_b200.h.
SIGNATURES = [
    ("elips_b200_status_string", c_char_p, [c_int]),
    ("elips_b200_device_count", c_int, [POINTER(c_int)]),
    ("elips_b200_device_error", c_int, [c_int, POINTER(c_int)]),
    ("elips_b200_wait_selftest", c_int, [c_int, c_uint64]),
    ("elips_b200_exact_create", c_int, [c_int, c_int, c_int, c_uint32, POINTER(c_void_p)]),
    ("elips_b200_exact_add", c_int, [c_void_p, c_void_p, c_size_t]),
    ("elips_b200_exact_add_device", c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    ("elips_b200_exact_size", c_int, [c_void_p, POINTER(c_size_t)]),
    ("elips_b200_exact_destroy", c_int, [c_void_p]),
    ("elips_b200_exact_search", c_int,
     [c_void_p, c_void_p, c_size_t, c_size_t, c_void_p, c_void_p, c_void_p]),
    ("elips_b200_exact_search_device", c_int,
     [c_void_p, c_void_p, c_size_t, c_size_t, c_void_p, c_void_p, c_void_p, c_void_p]),
    ("elips_b200_exact_search_noalloc", c_int,
     [c_void_p, c_void_p, c_size_t, c_size_t, c_void_p, c_void_p, c_void_p, c_void_p]),
    ("elips_b200_exact_search_candidates_device", c_int,
     [c_void_p, c_void_p, c_size_t, c_size_t, c_void_p, c_uint32, c_void_p, c_void_p]),
    ("elips_b200_merge_candidates_device", c_int,
     [c_int, c_void_p, c_size_t, c_size_t, c_size_t, c_int, c_void_p, c_void_p, c_void_p]),
    ("elips_b200_exact_search_candidates_shared_device", c_int, [c_void_p, c_void_p, c_size_t, c_size_t, c_void_p, c_uint32, c_void_p, c_void_p, c_void_p]),
    ("elips_b200_peer_alloc", c_int, [c_int, c_size_t, POINTER(c_void_p), c_void_p]),
    ("elips_b200_peer_open", c_int, [c_int, c_void_p, POINTER(c_void_p)]),
    ("elips_b200_peer_close", c_int, [c_int, c_void_p]),
    ("elips_b200_peer_free", c_int, [c_int, c_void_p]),
    ("elips_b200_copy_device", c_int, [c_int, c_void_p, c_void_p, c_size_t, c_void_p]),
    ("elips_b200_fill_device", c_int, [c_int, c_void_p, c_int, c_size_t, c_void_p]),
    ("elips_b200_compute_distances_batch", c_int,
     [c_int, c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_int, c_int, c_void_p]),
    ("elips_b200_top_k", c_int,
     [c_int, c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_int, c_void_p]),
    ("elips_b200_gemm_fp32", c_int,
     [c_int, c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_int, c_int, c_int, c_void_p]),
    ("elips_b200_quant_create", c_int,
     [c_int, c_int, c_int, c_uint32, c_uint32, c_uint32, c_void_p, c_void_p, POINTER(c_void_p)]),
    ("elips_b200_quant_add", c_int, [c_void_p, c_void_p, c_size_t]),
    ("elips_b200_quant_add_codes", c_int, [c_void_p, c_void_p, c_size_t]),
    ("elips_b200_quant_size", c_int, [c_void_p, POINTER(c_size_t)]),
    ("elips_b200_quant_search", c_int, [c_void_p, c_void_p, c_size_t, c_size_t, c_void_p, c_void_p]),
    ("elips_b200_quant_search_device", c_int,
     [c_void_p, c_void_p, c_size_t, c_size_t, c_void_p, c_void_p, c_void_p]),
    ("elips_b200_quant_destroy", c_int, [c_void_p]),
    ("elips_b200_exact_live", c_int, [c_void_p, POINTER(c_size_t)]),
    ("elips_b200_exact_device_bytes", c_int, [c_void_p, POINTER(c_size_t)]),
    ("elips_b200_exact_remove", c_int, [c_void_p, c_size_t, POINTER(c_int)]),
    ("elips_b200_exact_compact", c_int, [c_void_p, c_void_p, c_size_t]),
    ("elips_b200_exact_snapshot_bytes", c_int, [c_void_p, POINTER(c_size_t)]),
    ("elips_b200_exact_export", c_int, [c_void_p, c_void_p, c_size_t]),
    ("elips_b200_exact_import", c_int, [c_void_p, c_void_p, c_size_t]),
    ("elips_b200_ivfpq_export", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    ("elips_b200_ivfflat_export", c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
    ("elips_b200_batcher_create", c_int, [c_void_p, c_size_t, c_size_t, POINTER(c_void_p)]),
    ("elips_b200_batcher_search", c_int, [c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    ("elips_b200_batcher_stats", c_int, [c_void_p, POINTER(c_uint64), POINTER(c_uint64)]),
    ("elips_b200_batcher_flush", c_int, [c_void_p]),
    ("elips_b200_batcher_pending", c_int, [c_void_p, POINTER(c_uint64)]),
    ("elips_b200_batcher_destroy", c_int, [c_void_p]),
    ("elips_b200_ivfpq_probe_device", c_int, [c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    ("elips_b200_ivfpq_search_candidates_probed_device", c_int,
     [c_void_p, c_void_p, c_size_t, c_size_t, c_void_p, c_void_p, c_void_p]),
    ("elips_b200_ivfpq_search_candidates_shared_device", c_int,
     [c_void_p, c_void_p, c_size_t, c_size_t, c_void_p, c_void_p, c_void_p, c_void_p]),
    ("elips_b200_ivfpq_remove", c_int, [c_void_p, c_size_t]),
    ("elips_b200_ivfpq_rebuild_codes", c_int, [c_void_p]),
    ("elips_b200_ivfflat_remove", c_int, [c_void_p, c_size_t]),
    ("elips_b200_normalize_rows", c_int, [c_int, c_void_p, c_void_p, c_size_t, c_size_t, c_int, c_void_p]),
    ("elips_b200_kmeans", c_int, [c_int, c_void_p, c_size_t, c_size_t, c_size_t, c_size_t, c_void_p, c_int, c_void_p]),
    ("elips_b200_train_pq_codebook", c_int,
     [c_int, c_void_p, c_size_t, c_size_t, c_size_t, c_size_t, c_size_t, c_void_p, c_int, c_void_p]),
    ("elips_b200_ivf_assign", c_int,
     [c_int, c_int, c_void_p, c_size_t, c_size_t, c_void_p, c_size_t, c_void_p, c_void_p, c_int, c_void_p]),
    ("elips_b200_ivf_train", c_int,
     [c_int, c_int, c_void_p, c_size_t, c_size_t, c_size_t, c_size_t, c_void_p, c_void_p, c_int, c_void_p]),
    ("elips_b200_ivfpq_train", c_int,
     [c_int, c_int, c_void_p, c_size_t, c_size_t, c_size_t, c_size_t, c_size_t, c_uint32, c_void_p, c_void_p,
      c_void_p, c_void_p, c_int, c_void_p]),
    ("elips_b200_ivfpq_create", c_int,
     [c_int, c_int, c_uint32, c_uint32, c_uint32, c_uint32, c_uint32, c_void_p, c_void_p, POINTER(c_void_p)]),
    ("elips_b200_ivfpq_add", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_size_t]),
    ("elips_b200_ivfpq_add_device", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    ("elips_b200_ivfpq_size", c_int, [c_void_p, POINTER(c_size_t)]),
    ("elips_b200_ivfpq_set_nprobe", c_int, [c_void_p, c_uint32]),
    ("elips_b200_ivfpq_search", c_int, [c_void_p, c_void_p, c_size_t, c_size_t, c_void_p, c_void_p]),
    ("elips_b200_ivfpq_search_device", c_int,
     [c_void_p, c_void_p, c_size_t, c_size_t, c_void_p, c_void_p, c_void_p]),
    ("elips_b200_ivfpq_codes_device", c_int, [c_void_p, c_void_p, c_void_p]),
    ("elips_b200_ivfpq_set_list_range", c_int, [c_void_p, c_uint32, c_uint32]),
    ("elips_b200_ivfpq_set_owned_lists", c_int, [c_void_p, c_void_p, c_size_t]),
    ("elips_b200_ivfpq_search_candidates_device", c_int, [c_void_p, c_void_p, c_size_t, c_size_t, c_void_p, c_void_p]),
    ("elips_b200_ivfpq_rerank_device", c_int,
     [c_void_p, c_void_p, c_size_t, c_size_t, c_void_p, c_void_p, c_void_p, c_void_p]),
    ("elips_b200_ivfpq_destroy", c_int, [c_void_p]),
    ("elips_b200_ivfflat_create", c_int,
     [c_int, c_int, c_uint32, c_uint32, c_uint32, c_void_p, POINTER(c_void_p)]),
    ("elips_b200_ivfflat_add", c_int, [c_void_p, c_void_p, c_void_p, c_size_t]),
    ("elips_b200_ivfflat_add_device", c_int, [c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    ("elips_b200_ivfflat_size", c_int, [c_void_p, POINTER(c_size_t)]),
    ("elips_b200_ivfflat_set_nprobe", c_int, [c_void_p, c_uint32]),
    ("elips_b200_ivfflat_search", c_int, [c_void_p, c_void_p, c_size_t, c_size_t, c_void_p, c_void_p]),
    ("elips_b200_ivfflat_search_device", c_int,
     [c_void_p, c_void_p, c_size_t, c_size_t, c_void_p, c_void_p, c_void_p]),
    ("elips_b200_ivfflat_destroy", c_int, [c_void_p]),
    ("elips_b200_profiler_enable", c_int, [c_int]),
    ("elips_b200_profiler_stats", c_int,
     [c_char_p, POINTER(ctypes.c_uint64), POINTER(ctypes.c_double), POINTER(ctypes.c_uint64)]),
    ("elips_b200_profiler_reset", c_int, []),
    ("elips_b200_launch_count", c_int, [POINTER(ctypes.c_uint64)]),
]


class ElipsB200Error(RuntimeError):
    """A non-zero status from the C ABI. `status` is the ELIPS_B200_* code."""

    def __init__(self, status: int, where: str):
        self.status = status
        super().__init__(f"{where}: {status_name(status)} ({status})")


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is not built; run `python elips_b200/build.py` "
            "(the search path has no CPU fallback)")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, restype, argtypes in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


LIB = _load()


def status_name(status: int) -> str:
    return LIB.elips_b200_status_string(int(status)).decode()


def check(status: int, where: str) -> None:
    if status != OK:
        raise ElipsB200Error(status, where)


def device_count() -> int:
    n = c_int(0)
    status = LIB.elips_b200_device_count(ctypes.byref(n))
    if status not in (OK, DEVICE_NOT_FOUND, BACKEND_UNAVAILABLE):
        check(status, "elips_b200_device_count")
    return n.value


def device_error(device: int) -> int:
    code = c_int(0)
    check(LIB.elips_b200_device_error(device, ctypes.byref(code)), "elips_b200_device_error")
    return code.value


def profiler_enable(on: bool = True) -> None:
    check(LIB.elips_b200_profiler_enable(1 if on else 0), "elips_b200_profiler_enable")


def profiler_reset() -> None:
    check(LIB.elips_b200_profiler_reset(), "elips_b200_profiler_reset")


def profiler_stats(kernel: str | None = None) -> dict:
    """{'launches', 'total_ms', 'items'} for one kernel (None = all)."""
    n, ms, it = ctypes.c_uint64(0), ctypes.c_double(0.0), ctypes.c_uint64(0)
    check(LIB.elips_b200_profiler_stats(kernel.encode() if kernel else None, ctypes.byref(n),
                                        ctypes.byref(ms), ctypes.byref(it)), "elips_b200_profiler_stats")
    return {"launches": n.value, "total_ms": ms.value, "items": it.value}


def launch_count() -> int:
    n = ctypes.c_uint64(0)
    check(LIB.elips_b200_launch_count(ctypes.byref(n)), "elips_b200_launch_count")
    return n.value


__all__ = [n for n in dir() if not n.startswith("_")]
