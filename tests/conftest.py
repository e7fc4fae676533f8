"""Shared test setup: the `gpu` marker, the package import and golden-vector loading.

Tests marked `gpu` need an sm_100 device and call the kernels through the C ABI;
everything else runs on a CPU-only host (`pytest -m "not gpu"`).
"""
import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# The package directory is `gemma-npu_b200`; importing it registers `gemma_npu_b200`.
importlib.import_module("gemma-npu_b200")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU; runs the CUDA kernels")


def load_golden(name):
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def golden():
    return load_golden


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability()
    if (major, minor) != (10, 0):
        pytest.skip(f"kernels are built for sm_100a; device is sm_{major}{minor}")
    return torch.device("cuda", torch.cuda.current_device())
