import os
import sys

import pytest

# PyTorch (test plumbing: gloo process groups, device buffers) is imported before libwindlass_cuda loads NCCL on
# first tensor-parallel use, so that both share PyTorch's NCCL rather than the library pulling in the system copy
# first and PyTorch then failing to find its newer symbols in it.
try:
    import torch  # noqa: F401
except ImportError:
    pass

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def oracle():
    """The CPU oracle (built from oracle/*.c if its library is missing)."""
    from oracle import oracle as O
    O.lib()
    return O


@pytest.fixture(scope="session")
def wl():
    """libwindlass_cuda via ctypes; built in-tree if missing (no fallback when it cannot load)."""
    from windlass_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        from windlass_b200 import build
        build.build()
    _lib.lib()
    return _lib


@pytest.fixture(scope="session")
def tmpdir_session(tmp_path_factory):
    return tmp_path_factory.mktemp("windlass")


@pytest.fixture(scope="session")
def golden():
    import json
    with open(os.path.join(ROOT, "tests", "golden", "llamacpp_reference.json")) as f:
        return json.load(f)
