"""Launch overlap (programmatic dependent launch) keeps stream order: chains
of launches in which every kernel reads what the one ahead of it wrote give
the same bits with the overlap on (the default) and off.  A kernel that read
before the kernel ahead had finished would lose increments of the in-place
chain or read stale rows of the mixed one."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from test_parity_gpu import assert_same_f32, dev, host

pytestmark = pytest.mark.gpu


def add_chain(v7g, x0, y, steps):
    x = x0.clone()
    for _ in range(steps):
        v7g.add_inplace(x, y)  # each launch reads the previous launch's x
    torch.cuda.synchronize()
    return host(x)


def mixed_chain(v7g, r0, d, w, wq, ws):
    """add + RMSNorm -> RMSNorm -> Q8 -> SwiGLU -> Q8 GEMV, four rounds, each
    launch consuming the output of the one before it."""
    r = r0.clone()
    o = torch.empty_like(r)
    g = torch.empty_like(r)
    codes = torch.empty(r.shape, dtype=torch.int8, device=r.device)
    scales = torch.empty(r.shape[0], r.shape[1] // 64, device=r.device)
    y = torch.empty(8, wq.shape[0], device=r.device)
    for _ in range(4):
        v7g.fused_add_rmsnorm_rows(o, r, d, w, 1e-6)
        v7g.rmsnorm_quantize_rows(codes, scales, o, w, 1e-6)
        v7g.swiglu(g, o, r)
        v7g.add_inplace(r, g)
        v7g.q8_gemv(y, codes[:8], scales[:8], wq, ws)
    torch.cuda.synchronize()
    return host(r), host(o), host(codes), host(scales), host(y)


def test_overlap_switch_default_on(cuda):
    import v7multiplikator_b200 as v7g
    assert v7g.launch_overlap()


@pytest.mark.parametrize("rows,n", [(4096, 2048), (3, 64)])
def test_dependent_add_chain_same_bits(cuda, oracle, rows, n):
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(rows + n)
    x0 = rng.standard_normal((rows, n), dtype=np.float32)
    y = rng.standard_normal((rows, n), dtype=np.float32)
    steps = 50
    try:
        v7g.set_launch_overlap(True)
        on = add_chain(v7g, dev(x0), dev(y), steps)
        v7g.set_launch_overlap(False)
        off = add_chain(v7g, dev(x0), dev(y), steps)
    finally:
        v7g.set_launch_overlap(True)
    assert np.array_equal(on.view(np.uint32), off.view(np.uint32))
    ref = x0.copy()
    for _ in range(steps):
        ref = oracle.add_inplace(ref, y)
    assert_same_f32(on, ref)


def test_dependent_mixed_chain_same_bits(cuda):
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(11)
    rows, n, d = 1024, 2048, 512
    r0 = dev(rng.standard_normal((rows, n), dtype=np.float32))
    dd = dev((0.5 * rng.standard_normal((rows, n))).astype(np.float32))
    w = dev((1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32))
    wq = dev(rng.integers(-127, 128, (d, n), dtype=np.int8))
    ws = dev((0.001 + 0.01 * rng.random((d, n // 64))).astype(np.float32))
    try:
        v7g.set_launch_overlap(True)
        on = mixed_chain(v7g, r0, dd, w, wq, ws)
        v7g.set_launch_overlap(False)
        off = mixed_chain(v7g, r0, dd, w, wq, ws)
    finally:
        v7g.set_launch_overlap(True)
    for a, b in zip(on, off):
        assert a.shape == b.shape
        assert np.array_equal(a.view(np.uint8), b.view(np.uint8))
