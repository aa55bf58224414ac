"""Reference-surface entries (Microsoft x64 convention, no stream argument)
given DEVICE pointers: the call must see inputs that the caller's own queued
work is still writing on another stream, and must leave the caller's current
device as it was.  Checked against the oracle bit for bit."""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
F = np.float32
ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def shim(tmp_path_factory):
    so = tmp_path_factory.mktemp("shim") / "libmsabi_shim.so"
    subprocess.run(["gcc", "-O1", "-shared", "-fPIC", str(ROOT / "tests" / "msabi_shim.c"), "-o", str(so)], check=True)
    s = ctypes.CDLL(str(so))
    s.shim_v7s_rmsnorm.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int]
    s.shim_v7s_add_inplace.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int]
    return s


def entry(name: str) -> int:
    import v7multiplikator_b200 as v7g
    return ctypes.cast(getattr(v7g.lib(), name), ctypes.c_void_p).value


def test_device_inputs_written_on_another_stream(cuda, oracle, shim):
    import v7multiplikator_b200 as v7g
    n = 2048
    rng = np.random.default_rng(11)
    src_h = rng.normal(0, 1, n).astype(F)
    w_h = rng.normal(1, 0.1, n).astype(F)
    src, w = torch.from_numpy(src_h).cuda(), torch.from_numpy(w_h).cuda()
    x = torch.zeros(n, device=cuda)
    o = torch.full((n,), float("nan"), device=cuda)
    v7g.set_rms_eps(1e-6)
    torch.cuda.synchronize()
    side = torch.cuda.Stream(device=cuda)
    with torch.cuda.stream(side):
        torch.cuda._sleep(100_000_000)  # about 50 ms: x is written long after the call below starts
        x.copy_(src)
    shim.shim_v7s_rmsnorm(entry("v7s_rmsnorm"), o.data_ptr(), x.data_ptr(), w.data_ptr(), n)
    assert side.query(), "the call returned before the caller's queued work on another stream had finished"
    assert not v7g.lib().v7_engine_is_dead()
    got = o.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), oracle.rmsnorm(src_h[None], w_h, 1e-6)[0].view(np.uint32))

    # in place: y written on the side stream, x += y through the reference entry
    y = torch.zeros(n, device=cuda)
    torch.cuda.synchronize()
    with torch.cuda.stream(side):
        torch.cuda._sleep(100_000_000)
        y.copy_(src)
    shim.shim_v7s_add_inplace(entry("v7s_add_inplace"), x.data_ptr(), y.data_ptr(), n)
    assert np.array_equal(x.cpu().numpy(), oracle.add_inplace(src_h.copy(), src_h))


def test_caller_device_is_kept(cuda, oracle, shim):
    """Pointers on another GPU (where there is one): the call selects that
    device for its work and restores the caller's afterwards."""
    import v7multiplikator_b200 as v7g
    n = 256
    rng = np.random.default_rng(12)
    x_h = rng.normal(0, 1, n).astype(F)
    w_h = rng.normal(1, 0.1, n).astype(F)
    dev = torch.device("cuda", 1) if torch.cuda.device_count() > 1 else cuda
    x, w = torch.from_numpy(x_h).to(dev), torch.from_numpy(w_h).to(dev)
    o = torch.empty(n, device=dev)
    v7g.set_rms_eps(1e-6)
    torch.cuda.set_device(0)
    torch.cuda.synchronize(dev)
    shim.shim_v7s_rmsnorm(entry("v7s_rmsnorm"), o.data_ptr(), x.data_ptr(), w.data_ptr(), n)
    assert torch.cuda.current_device() == 0
    got = o.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), oracle.rmsnorm(x_h[None], w_h, 1e-6)[0].view(np.uint32))
