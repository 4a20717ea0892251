import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def _cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def lib():
    from minixla_b200 import lib as mlib

    return mlib.load()


@pytest.fixture(scope="session")
def gpu_ctx(lib):
    if not _cuda_available():
        pytest.skip("no CUDA device")
    ctx = lib.gpu_ctx_create()
    assert ctx, f"gpu_ctx_create failed: {lib.mxb_last_error()}"
    yield ctx
    lib.gpu_ctx_destroy(ctx)


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return np.load(Path(__file__).resolve().parent / "golden" / "golden.npz")


@pytest.fixture(scope="session")
def host_threads():
    return os.cpu_count() or 1
