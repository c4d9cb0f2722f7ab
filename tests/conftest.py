import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) CUDA device")


def load_build_module():
    """elips_b200/build.py loaded by path (importing the package would load the
    library it builds)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("elips_b200_build", ROOT / "elips_b200" / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session", autouse=True)
def _built_library():
    """Builds the CUDA library and the CPU checkers when they are missing or
    stale (nvcc cross-compiles here; on a GPU box the shipped build is used)."""
    b = load_build_module()
    if b.needs_build():
        b.build()
    import oracle
    oracle.build(ref=True)
    yield


def pytest_collection_modifyitems(config, items):
    if _cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def nthreads():
    return os.cpu_count() or 1
