import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")
    # the oracle is a few C files: build it if this checkout has not yet (the GPU box gets the prebuilt .so)
    if not os.path.exists(os.path.join(ROOT, "oracle", "liboracle.so")):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "oracle"], check=True)


@pytest.fixture(scope="session")
def golden():
    return GOLDEN


@pytest.fixture(scope="session")
def cuda_dev():
    """torch on cuda:0 plus the native library bound to the same device"""
    import torch

    import quillm_b200 as qb

    assert torch.cuda.is_available(), "GPU test without a CUDA device"
    torch.cuda.set_device(0)
    qb.check(qb.cuda().qmc_set_device(0), "set_device")
    return torch.device("cuda:0")
