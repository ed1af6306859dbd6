"""Test configuration: puts the package and the oracle on sys.path and
registers the `gpu` marker (tests that need a B200)."""

import os
import pathlib
import sys

ROOT = pathlib.Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "gpt-speedrun-tpu_b200"))
sys.path.insert(0, str(ROOT))

import pytest  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    from rig_b200 import _lib

    _lib.load()
    return torch.device("cuda", 0)
