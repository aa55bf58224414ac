"""Shared fixtures.  GPU tests carry @pytest.mark.gpu; everything else runs on
the CPU (oracle against the reference's golden outputs, C-ABI exports, host
logic, multi-rank gloo)."""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
TESTS = Path(__file__).resolve().parent
if str(TESTS) not in sys.path:
    sys.path.insert(0, str(TESTS))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device of compute capability 10.x (B200)")


@pytest.fixture(scope="session")
def oracle():
    from oracle.pyoracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def native_lib_path():
    from v7multiplikator_b200 import build
    if not build.LIB.exists():
        build.build()
    return build.LIB


@pytest.fixture(scope="session")
def golden():
    return np.load(TESTS / "golden" / "kt_cref.npz")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.skip("needs an sm_100 device")
    import v7multiplikator_b200 as v7g
    v7g.lib()
    return torch.device("cuda:0")


def run(cmd, **kw):
    return subprocess.run(cmd, capture_output=True, text=True, **kw)
