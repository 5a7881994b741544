import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import __graft_entry__  # noqa: E402

pai = __graft_entry__.load_package()
ORACLE_LIB = ROOT / "oracle" / "build" / "liboracle.so"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (runs the sm_100a kernels)")


def _has_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


HAS_GPU = _has_gpu()


def pytest_collection_modifyitems(config, items):
    if HAS_GPU:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def oracle_lib():
    from projectai_b200.cabi import NativeLibrary

    if not ORACLE_LIB.exists():
        __graft_entry__.build_oracle()
    return NativeLibrary(ORACLE_LIB, "oracle_")


@pytest.fixture()
def oracle(oracle_lib):
    from projectai_b200.cabi import NativeBackend

    be = NativeBackend(oracle_lib)
    yield be
    be.close()


@pytest.fixture(scope="session")
def cuda_lib():
    return pai.cuda_library()


@pytest.fixture()
def cuda(cuda_lib):
    from projectai_b200.cabi import NativeBackend

    be = NativeBackend(cuda_lib, int(os.environ.get("PAI_TEST_DEVICE", "0")))
    yield be
    be.close()
