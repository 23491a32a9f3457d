import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; runs the CUDA path through the C ABI")


def cuda_ok() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def orc():
    import oracle

    return oracle


@pytest.fixture(scope="session")
def gpu_ctx():
    if not cuda_ok():
        pytest.skip("no CUDA device")
    import deepseek_cpp_infer_b200 as dsb

    ctx = dsb.Context(0)
    # torch makes the inputs on its default stream: run the context there too
    ctx.use_legacy_stream()
    yield ctx
    ctx.close()
