"""v7g_rmsnorm_rows_noalloc: RMSNorm on host buffers for callers that must not
have a library allocate device memory (a process whose framework allocator
already holds the GPU's memory, a loop that cannot take the synchronisation
cudaMalloc / cudaFree bring, a deployment that forbids allocation after
start-up).  Its staging lives in a static device array of fixed size.

Checked through the C-ABI (ctypes, host numpy buffers), bit for bit -- the bar
every parity test here uses -- against the CPU oracle (the restatement of the
reference's rmsnorm_kernel.inc) and against the existing v7g_rmsnorm_rows on
device tensors, on calls in a row whose sizes differ, so nothing left in the
shared array from one call can reach the next.  A request beyond the array's
size is refused without touching the output, and a stream of another device
is refused.  This file is collected last so that a run stopping at its first
failure has run everything else."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
F = np.float32


def existing_entry(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    import v7multiplikator_b200 as v7g
    out = torch.empty(x.shape, device="cuda")
    v7g.rmsnorm_rows(out, torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), eps)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def call_noalloc(o: np.ndarray, x: np.ndarray, w: np.ndarray, eps: float, stream=None) -> int:
    import v7multiplikator_b200 as v7g
    fn = v7g.lib().v7g_rmsnorm_rows_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float,
                   ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn(o.ctypes.data, x.ctypes.data, w.ctypes.data, x.shape[0], x.shape[1], eps, stream)


def same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    return np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_noalloc_matches_oracle_and_existing_entry_on_calls_in_a_row(cuda, oracle):
    rng = np.random.default_rng(2024)
    cases = [(64, 2048, 1e-6), (5, 96, 1e-5), (200, 1024, 1e-6), (64, 2048, 1e-6)]
    for rows, n, eps in cases:
        x = rng.normal(0, 1, (rows, n)).astype(F)
        w = rng.normal(1, 0.1, n).astype(F)
        o = np.full((rows, n), np.nan, F)
        assert call_noalloc(o, x, w, eps) == 0
        assert same_bits(o, oracle.rmsnorm(x, w, eps)), (rows, n)
        assert same_bits(o, existing_entry(x, w, eps)), (rows, n)


def test_noalloc_refuses_work_beyond_its_array(cuda, oracle):
    import v7multiplikator_b200 as v7g
    n = 2048
    rows = v7g.ops.NOALLOC_SCRATCH_BYTES // (2 * 4 * n) + 1  # x and o no longer fit
    x = np.ones((rows, n), F)
    w = np.ones(n, F)
    o = np.full((rows, n), 7.0, F)
    assert call_noalloc(o, x, w, 1e-6) == v7g.ops.V7G_ERR_ARG
    assert b"static scratch" in v7g.lib().v7g_last_error()
    assert (o == 7.0).all()
    # and the largest fitting request still works, through the Python wrapper
    rows = (v7g.ops.NOALLOC_SCRATCH_BYTES - 4 * n) // (2 * 4 * n)
    x = np.random.default_rng(1).normal(0, 1, (rows, n)).astype(F)
    o = np.empty_like(x)
    v7g.rmsnorm_rows_noalloc(o, x, w, 1e-6)
    assert same_bits(o, oracle.rmsnorm(x, w, 1e-6))


def test_noalloc_on_a_caller_stream(cuda, oracle):
    """A caller's own stream of the current device is accepted; one of another
    device (where there is one) is refused before anything is queued."""
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(7)
    x = rng.normal(0, 1, (32, 512)).astype(F)
    w = rng.normal(1, 0.1, 512).astype(F)
    s = torch.cuda.Stream(device=0)
    o = np.empty_like(x)
    assert call_noalloc(o, x, w, 1e-6, s.cuda_stream) == 0
    assert same_bits(o, oracle.rmsnorm(x, w, 1e-6))
    if torch.cuda.device_count() > 1:
        other = torch.cuda.Stream(device=1)
        o = np.full_like(x, 3.0)
        assert call_noalloc(o, x, w, 1e-6, other.cuda_stream) == v7g.ops.V7G_ERR_ARG
        assert b"belongs to device" in v7g.lib().v7g_last_error()
        assert (o == 3.0).all()
