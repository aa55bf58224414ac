"""v7g_rmsnorm_rows_noalloc: RMSNorm on host buffers for callers that must not
have a library allocate device memory (a process whose framework allocator
already holds the GPU's memory, a loop that cannot take the synchronisation
cudaMalloc / cudaFree bring, a deployment that forbids allocation after
start-up).  Its staging lives in a static device array of fixed size.

Checked through the C-ABI (ctypes, host numpy buffers) against the existing
v7g_rmsnorm_rows on device tensors, bit for bit -- the bar every parity test
here uses -- on calls in a row whose sizes differ, so nothing left in the
shared array from one call can reach the next; and a request beyond the
array's size is refused without touching the output.  This file is collected
last so that a run stopping at its first failure has run everything else."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
F = np.float32


def reference(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    import v7multiplikator_b200 as v7g
    out = torch.empty(x.shape, device="cuda")
    v7g.rmsnorm_rows(out, torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), eps)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def call_noalloc(o: np.ndarray, x: np.ndarray, w: np.ndarray, eps: float) -> int:
    import v7multiplikator_b200 as v7g
    fn = v7g.lib().v7g_rmsnorm_rows_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float,
                   ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn(o.ctypes.data, x.ctypes.data, w.ctypes.data, x.shape[0], x.shape[1], eps, None)


def test_noalloc_matches_existing_entry_on_calls_in_a_row(cuda):
    rng = np.random.default_rng(2024)
    cases = [(64, 2048, 1e-6), (5, 96, 1e-5), (200, 1024, 1e-6)]
    for rows, n, eps in cases:
        x = rng.normal(0, 1, (rows, n)).astype(F)
        w = rng.normal(1, 0.1, n).astype(F)
        o = np.full((rows, n), np.nan, F)
        assert call_noalloc(o, x, w, eps) == 0
        want = reference(x, w, eps)
        assert np.array_equal(o.view(np.uint32), want.view(np.uint32)), (rows, n)


def test_noalloc_refuses_work_beyond_its_array(cuda):
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
    assert np.array_equal(o, reference(x, w, 1e-6))
