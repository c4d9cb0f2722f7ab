"""The C-ABI library loads and exports every entry point include/elips_b200.h
declares (no compute calls: this runs without a GPU)."""
import ctypes
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "elips_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(elips_b200_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "elips_b200_exact_search" in names
    assert len(names) >= 10


def test_library_exports_every_declared_symbol():
    from elips_b200 import _capi
    lib = ctypes.CDLL(str(_capi.LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_binding_table_matches_header():
    from elips_b200 import _capi
    bound = {name for name, _, _ in _capi.SIGNATURES}
    assert bound == set(declared_functions())


def test_status_strings_and_error_mapping():
    from elips_b200 import _capi
    # 1..8 mirror elips::gpu::GpuError (GpuPort.hpp:15-24) in order.
    expected = ["DeviceNotFound", "InsufficientMemory", "KernelLaunchFailed", "TransferFailed",
                "IndexBuildFailed", "UnsupportedMetric", "InitializationFailed", "BackendUnavailable"]
    assert [_capi.status_name(i) for i in range(1, 9)] == expected
    assert _capi.status_name(0) == "Ok"
    assert _capi.status_name(9) == "DimensionMismatch"


def test_null_arguments_are_rejected_without_a_device():
    from elips_b200 import _capi
    assert _capi.LIB.elips_b200_exact_create(0, 0, 0, 8, None) == _capi.INVALID_ARGUMENT
    assert _capi.LIB.elips_b200_exact_add(None, None, 0) == _capi.INVALID_ARGUMENT
    assert _capi.LIB.elips_b200_exact_search(None, None, 1, 1, None, None, None) == _capi.INVALID_ARGUMENT
    assert _capi.LIB.elips_b200_merge_candidates_device(0, None, 1, 1, 1, 7, None, None, None) == \
        _capi.UNSUPPORTED_METRIC


def test_library_links_no_torch():
    """The shipped library depends on the CUDA runtime only (statically)."""
    import subprocess
    from elips_b200 import _capi
    out = subprocess.run(["readelf", "-d", str(_capi.LIB_PATH)], capture_output=True, text=True, check=True).stdout
    needed = re.findall(r"\(NEEDED\)\s+Shared library: \[([^\]]+)\]", out)
    assert needed, out
    assert not [n for n in needed if "torch" in n or "c10" in n or "cudart" in n], needed
