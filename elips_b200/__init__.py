"""B200-native k-NN search backend for ELIPS.

The compute path is hand-written sm_100a CUDA in elips_b200/csrc, built into
elips_b200/libelips_b200.so and reached through the C ABI declared in
include/elips_b200.h. Importing this package loads that library and raises if
it is missing: there is no CPU fallback.
"""
from . import _capi
from ._capi import ElipsB200Error, device_count, status_name
from .exact import DimensionMismatch, DynamicBatcher, ExactIndex, merge_candidates_device

__all__ = ["ElipsB200Error", "DimensionMismatch", "DynamicBatcher", "ExactIndex", "merge_candidates_device",
           "device_count", "status_name"]
