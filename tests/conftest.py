"""Shared fixtures. GPU tests carry ``@pytest.mark.gpu`` and call the CUDA
library through its C ABI; CPU tests cover the oracle, host logic and the ABI
surface (load + exported symbols) without a GPU."""
import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

PKG = "sd-vulkan-pixel10-tensor-g5_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


def load_pkg():
    return importlib.import_module(PKG)


@pytest.fixture(scope="session")
def sdg():
    return load_pkg()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.manual_seed(0)
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def unet_weights():
    """Seeded default-init SD1.5 UNet weights (fp16, PyTorch layout)."""
    from oracle import weights as W
    return W.make_weights(0)


@pytest.fixture(scope="session")
def engine(sdg, cuda, unet_weights):
    from oracle import weights as W
    e = sdg.Engine(0)
    e.upload_weights(W.iter_reference_blobs(unet_weights))
    e.prepare()
    yield e
    e.release()
