import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# The reference checkout, when present (BLOCKLAB_REFERENCE_DIR, else its usual location here).
REFERENCE = os.environ.get("BLOCKLAB_REFERENCE_DIR", "/root/reference")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle

    return Oracle()


@pytest.fixture(scope="session")
def ref_cpu():
    from oracle.oracle import Reference, ref_available

    if not ref_available("cpu"):
        pytest.skip("reference CPU build (oracle/_ref/libref_cpu.so) not built")
    return Reference("cpu")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
