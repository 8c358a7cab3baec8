import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def bf16_bits(x):
    from oracle.oracle import bf16_bits as _b
    return _b(x)


def bf16_to_f32(b):
    from oracle.oracle import bf16_to_f32 as _f
    return _f(b)


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    from c_gpt2_b200 import ops
    ops.init(0)
    return torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _device_error_clean(request):
    """Every GPU test must leave the device error word at zero."""
    yield
    if request.node.get_closest_marker("gpu") is not None:
        from c_gpt2_b200 import ops
        assert ops.device_error(reset=True) == 0, "a kernel recorded a device error"
