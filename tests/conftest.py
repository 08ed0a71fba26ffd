"""Shared test setup: the ``gpu`` marker, import paths and fixture loading."""

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "comfyui-solattn_triton_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(REPO), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100) device")


def load_golden(name):
    return np.load(GOLDEN / f"{name}.npz")


def golden_meta(g):
    B, T, H, D, blk = (int(x) for x in g["meta"])
    return B, T, H, D, blk


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.skip("kernels are built for sm_100a only")
    return torch.device("cuda:0")


# GPU tests read each call's device error word (bounded-wait timeouts surface as
# RuntimeError instead of silently wrong output).
import os as _os
_os.environ.setdefault("SOLB200_SYNC_CHECK", "1")
