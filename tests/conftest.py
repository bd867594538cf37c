"""Shared pytest setup: markers, import paths and golden-fixture loaders."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_moe_fixture(name: str = "moe_fixture.safetensors"):
    """The reference's golden tensors (tests/golden/<name>) as numpy; bf16 tensors come back
    as uint16 bit patterns, uint32 as uint32."""
    import torch
    from safetensors.torch import load_file

    out = {}
    for k, v in load_file(os.path.join(GOLDEN, name)).items():
        if v.dtype == torch.bfloat16:
            out[k] = v.view(torch.int16).numpy().view(np.uint16).copy()
        elif v.dtype == torch.uint32:
            out[k] = v.view(torch.int32).numpy().view(np.uint32).copy()
        else:
            out[k] = v.numpy().copy()
    return out


@pytest.fixture(scope="session")
def moe_fixture():
    return load_moe_fixture()


@pytest.fixture(scope="session")
def hc_fixture():
    return load_moe_fixture("hc_fixture.safetensors")


@pytest.fixture(scope="session")
def lru_trace():
    return dict(np.load(os.path.join(GOLDEN, "lru_trace.npz")))
