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
    s.shim_q8_batch4.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
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


class Batch4Args(ctypes.Structure):
    """v7_q8_batch4_args (include/v7_threading.h; src/q8_batch4.h:29-38)."""
    _fields_ = [("out", ctypes.c_void_p * 4), ("xq", ctypes.c_void_p * 4), ("xs", ctypes.c_void_p * 4),
                ("wq", ctypes.c_void_p), ("ws", ctypes.c_void_p), ("n", ctypes.c_uint32), ("d", ctypes.c_uint32)]


@pytest.mark.parametrize("name", ["v7s_q8_batch4", "v7d_q8_batch4"])
@pytest.mark.parametrize("where", ["host", "device"])
def test_q8_batch4_entries(cuda, oracle, shim, name, where):
    """The four-token Q8 GEMV of the reference surface, bound by name: each
    token's output equals the oracle's one-token v7d_q8 bit for bit (-128
    weight bytes included), with the four tokens' pointers anywhere, on the
    host or on the device."""
    from test_oracle_gemv import q8_case
    from test_parity_gpu import assert_same_f32
    assert ctypes.sizeof(Batch4Args) == 120
    rng = np.random.default_rng(44 if where == "host" else 45)
    n, d = 1024, 300
    xq, xs, wq, ws = q8_case(rng, 4, n, d)
    wq[::7, 5::131] = -128
    outs = [np.full(d, np.nan, dtype=F) for _ in range(4)]
    keep = []
    if where == "host":
        xqs = [np.ascontiguousarray(xq[t]) for t in range(4)]
        xss = [np.ascontiguousarray(xs[t]) for t in range(4)]
        ptr = lambda a: a.ctypes.data
        ins = xqs + xss + [wq, ws]
        out_p = [ptr(o) for o in outs]
    else:
        tens = [torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in [*xq, *xs, wq, ws]]
        ins = tens
        ptr = lambda t: t.data_ptr()
        dev_outs = [torch.full((d,), float("nan"), device=cuda) for _ in range(4)]
        out_p = [o.data_ptr() for o in dev_outs]
        keep = dev_outs
    args = Batch4Args()
    for t in range(4):
        args.out[t] = out_p[t]
        args.xq[t] = ptr(ins[t])
        args.xs[t] = ptr(ins[4 + t])
    args.wq, args.ws, args.n, args.d = ptr(ins[8]), ptr(ins[9]), n, d
    shim.shim_q8_batch4(entry(name), ctypes.byref(args))  # outputs start as NaN: a failed call cannot pass
    if where == "device":
        outs = [o.cpu().numpy() for o in keep]
    for t in range(4):
        assert_same_f32(outs[t][None], oracle.q8_gemv(xq[t:t + 1], xs[t:t + 1], wq, ws), f"{name} token {t}")
