"""The Q8-weight GEMVs on the GPU, through the C-ABI, bit for bit against the
oracle: v7d_q8, v7d_q8_fused, v7d_swiglu_q8 and v7d_swiglu (dual-row
arithmetic), at the reference validators' model shapes, ragged row counts,
batches, and the contract's edges (-128 weights, extreme scales, NaN/inf in
the fp32 activation of the fused quantiser)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from test_parity_gpu import assert_same_f32, dev, host
from test_oracle_gemv import q8_case

pytestmark = pytest.mark.gpu
F = np.float32

SHAPES = [(1024, 3072), (2048, 8192), (576, 1536), (960, 2560), (896, 4864), (64, 1), (128, 37), (4096, 100)]


def ref_fill(rng, shape, dtype):
    """The validators' distributions: int8 in [-100, 100], floats 0.1 + k/1000."""
    if dtype == np.int8:
        return rng.integers(-100, 101, shape, dtype=np.int8)
    return (0.1 + rng.integers(0, 100, shape) / 1000).astype(F)


@pytest.mark.parametrize("n,d", SHAPES)
@pytest.mark.parametrize("batch", [1, 3])
def test_q8_gemv(cuda, oracle, n, d, batch):
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(n * 7 + d + batch)
    xq, xs, wq, ws = q8_case(rng, batch, n, d)
    out = torch.empty(batch, d, device=cuda)
    v7g.q8_gemv(out, dev(xq), dev(xs), dev(wq), dev(ws))
    assert_same_f32(host(out), oracle.q8_gemv(xq, xs, wq, ws))


@pytest.mark.parametrize("n,d", SHAPES)
def test_swiglu_q8_gemv(cuda, oracle, n, d):
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(n + 3 * d)
    xq, xs = ref_fill(rng, (1, n), np.int8), ref_fill(rng, (1, n // 64), F)
    gq, gs = ref_fill(rng, (d, n), np.int8), ref_fill(rng, (d, n // 64), F)
    uq, us = ref_fill(rng, (d, n), np.int8), ref_fill(rng, (d, n // 64), F)
    out = torch.empty(1, d, device=cuda)
    v7g.swiglu_q8_gemv(out, dev(xq), dev(xs), dev(gq), dev(gs), dev(uq), dev(us))
    with np.errstate(all="ignore"):
        assert_same_f32(host(out), oracle.swiglu_q8_gemv(xq, xs, gq, gs, uq, us))


@pytest.mark.parametrize("n,d", SHAPES)
def test_swiglu_f32q8_gemv(cuda, oracle, n, d):
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(n + 5 * d)
    x = ref_fill(rng, (2, n), F)
    gq, gs = ref_fill(rng, (d, n), np.int8), ref_fill(rng, (d, n // 64), F)
    uq, us = ref_fill(rng, (d, n), np.int8), ref_fill(rng, (d, n // 64), F)
    out = torch.empty(2, d, device=cuda)
    v7g.swiglu_f32q8_gemv(out, dev(x), dev(gq), dev(gs), dev(uq), dev(us))
    with np.errstate(all="ignore"):
        assert_same_f32(host(out), oracle.swiglu_f32q8_gemv(x, gq, gs, uq, us))


@pytest.mark.parametrize("n,d", [(2048, 8192), (64, 5), (1024, 1000)])
def test_q8_fused_gemv(cuda, oracle, n, d):
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(n + d)
    x = rng.normal(0, 2, (2, n)).astype(F)
    x[0, 5] = np.nan
    x[1, 70 % n] = np.inf
    x[1, 200 % n] = 1e-39
    _, _, wq, ws = q8_case(rng, 1, n, d)
    out = torch.empty(2, d, device=cuda)
    v7g.q8_fused_gemv(out, dev(x), dev(wq), dev(ws))
    with np.errstate(all="ignore"):
        assert_same_f32(host(out), oracle.q8_fused_gemv(x, wq, ws))


def test_q8_fused_gemv_unaligned_activation(cuda, oracle):
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(2)
    n, d = 256, 70
    x = rng.normal(0, 1, (1, n)).astype(F)
    _, _, wq, ws = q8_case(rng, 1, n, d)
    buf = torch.zeros(n + 1, device=cuda)
    xt = buf[1:].view(1, n)
    xt.copy_(dev(x))
    out = torch.empty(1, d, device=cuda)
    v7g.q8_fused_gemv(out, xt, dev(wq), dev(ws))
    assert_same_f32(host(out), oracle.q8_fused_gemv(x, wq, ws))


def test_gemv_neg128_weights_and_extreme_scales(cuda, oracle):
    """Outside the exporter's contract (-128 weights) the kernel still
    reproduces the reference's vpsignb product; scales spanning the fp32
    range exercise FTZ in the scale product and the accumulation."""
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(4)
    n, d = 512, 64
    xq = rng.integers(-128, 128, (1, n), dtype=np.int8)
    wq = rng.integers(-128, 128, (d, n), dtype=np.int8)
    wq[:, ::7] = -128
    xs = np.exp2(rng.integers(-70, 60, (1, n // 64))).astype(F)
    ws = np.exp2(rng.integers(-70, 60, (d, n // 64))).astype(F)
    ws[3, 2] = 1e-39
    out = torch.empty(1, d, device=cuda)
    v7g.q8_gemv(out, dev(xq), dev(xs), dev(wq), dev(ws))
    with np.errstate(all="ignore"):
        assert_same_f32(host(out), oracle.q8_gemv(xq, xs, wq, ws))
    out2 = torch.empty(1, d, device=cuda)
    v7g.swiglu_q8_gemv(out2, dev(xq), dev(xs), dev(wq), dev(ws), dev(wq[::-1].copy()), dev(ws[::-1].copy()))
    with np.errstate(all="ignore"):
        assert_same_f32(host(out2), oracle.swiglu_q8_gemv(xq, xs, wq, ws, wq[::-1], ws[::-1]))


@pytest.mark.parametrize("n,d", [(512, 64), (8192, 2048)])
def test_gemv_neg128_borrow_patterns(cuda, oracle, n, d):
    """The streaming kernel tests each weight word for -128 bytes as the
    zero-byte test of w ^ 0x80808080, a subtraction of 0x01010101 in which a
    borrow runs from one byte into the next: a 0x81 byte above a 0x00 byte
    (a near miss, which must get no correction), and a -128 byte above a
    0x00 byte or above a chain of them (which must be corrected).  Each
    pattern at a different byte position of the 4-byte words, in some rows
    and groups only, against a signed activation; every form of the
    streaming kernel."""
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(n + d)
    xq = rng.integers(-128, 128, (1, n), dtype=np.int8)
    wq = rng.integers(-127, 128, (d, n), dtype=np.int8)
    wq[wq == 0] = 1
    u = wq.view(np.uint8)
    for r in range(0, d, 3):
        for c in range(r % 5 * 4, n, 40):
            k = c + (r % 3)                      # byte 0, 1 or 2 of its word
            pattern = (r // 3) % 3
            if pattern == 0:
                u[r, k], u[r, k + 1] = 0x00, 0x81  # near miss: nothing to correct
            elif pattern == 1:
                u[r, k], u[r, k + 1] = 0x00, 0x80  # a -128 reached by the borrow
            elif k % 4 < 2:
                u[r, k], u[r, k + 1], u[r, k + 2] = 0x00, 0x00, 0x80
    xs = (0.001 + rng.random((1, n // 64)) * 0.02).astype(F)
    ws = (0.001 + rng.random((d, n // 64)) * 0.02).astype(F)
    out = torch.empty(1, d, device=cuda)
    v7g.q8_gemv(out, dev(xq), dev(xs), dev(wq), dev(ws))
    assert_same_f32(host(out), oracle.q8_gemv(xq, xs, wq, ws), "q8")
    x = rng.normal(0, 1, (1, n)).astype(F)
    out_f = torch.empty(1, d, device=cuda)
    v7g.q8_fused_gemv(out_f, dev(x), dev(wq), dev(ws))
    assert_same_f32(host(out_f), oracle.q8_fused_gemv(x, wq, ws), "q8 fused")
    uq, us = wq[::-1].copy(), ws[::-1].copy()
    out_s = torch.empty(1, d, device=cuda)
    v7g.swiglu_q8_gemv(out_s, dev(xq), dev(xs), dev(wq), dev(ws), dev(uq), dev(us))
    with np.errstate(all="ignore"):
        assert_same_f32(host(out_s), oracle.swiglu_q8_gemv(xq, xs, wq, ws, uq, us), "swiglu q8")


@pytest.mark.parametrize("n,d", [(64, 1), (576, 13), (1024, 3000), (2048, 5000), (8192, 2048)])
def test_gemv_stream_pipeline_and_direct_kernels_agree(cuda, oracle, n, d):
    """16-byte aligned weights and scales take the streaming kernel, aligned
    weights with 4-byte aligned scales the pipelined kernel, 4-byte aligned
    weights the direct-load kernel: all equal the oracle, and no wait gave up."""
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(n ^ d)
    xq, xs, gq, gs = q8_case(rng, 2, n, d)
    _, _, uq, us = q8_case(rng, 1, n, d)
    want = oracle.swiglu_q8_gemv(xq, xs, gq, gs, uq, us)
    want0 = oracle.q8_gemv(xq, xs, gq, gs)
    xf = rng.normal(0, 1, (2, n)).astype(F)
    want2 = oracle.swiglu_f32q8_gemv(xf, gq, gs, uq, us)
    before = v7g.pipeline_timeouts()

    def at(a, shift):
        """a copy of a on the device starting `shift` bytes into a fresh buffer"""
        t = dev(a)
        flat = t.reshape(-1).view(torch.int8)
        buf = torch.zeros(flat.numel() + 16, dtype=torch.int8, device=cuda)
        buf[shift:shift + flat.numel()].copy_(flat)
        return buf[shift:shift + flat.numel()].view(t.dtype).view(t.shape)

    for wshift, sshift in ((0, 0), (0, 4), (4, 0)):
        gt, ut = at(gq, wshift), at(uq, wshift)
        gst, ust = at(gs, sshift), at(us, sshift)
        tag = f"weights +{wshift} B, scales +{sshift} B"
        out = torch.empty(2, d, device=cuda)
        v7g.swiglu_q8_gemv(out, dev(xq), dev(xs), gt, gst, ut, ust)
        with np.errstate(all="ignore"):
            assert_same_f32(host(out), want, tag)
        out0 = torch.empty(2, d, device=cuda)
        v7g.q8_gemv(out0, dev(xq), at(xs, sshift), gt, gst)
        assert_same_f32(host(out0), want0, "q8, " + tag)
        # the fp32-activation kernel on the same weights, activation aligned or not
        for xshift in (0, 4):
            out2 = torch.empty(2, d, device=cuda)
            v7g.swiglu_f32q8_gemv(out2, at(xf, xshift), gt, gst, ut, ust)
            with np.errstate(all="ignore"):
                assert_same_f32(host(out2), want2, f"fp32 activation +{xshift} B, " + tag)
    assert v7g.pipeline_timeouts() == before == 0


def test_gemv_rejects_bad_shapes(cuda):
    import v7multiplikator_b200 as v7g
    x = torch.zeros(1, 96, dtype=torch.int8, device=cuda)
    w = torch.zeros(4, 96, dtype=torch.int8, device=cuda)
    s = torch.zeros(4, 1, device=cuda)
    with pytest.raises(v7g.V7GError, match="multiple of 64"):
        v7g.q8_gemv(torch.empty(1, 4, device=cuda), x, torch.zeros(1, 1, device=cuda), w, s)


def test_gemv_longest_rows(cuda, oracle):
    """The longest activation the entries accept (n = 65536, whose staged
    activation no longer fits the streaming kernel's layout, so the fallback
    paths run), a ragged d and two batch rows, all four products against the
    oracle; one group more is refused with the limit named."""
    import v7multiplikator_b200 as v7g
    n, d = 65536, 40
    rng = np.random.default_rng(65536)
    xq, xs, wq, ws = q8_case(rng, 2, n, d)
    out = torch.empty(2, d, device=cuda)
    v7g.q8_gemv(out, dev(xq), dev(xs), dev(wq), dev(ws))
    assert_same_f32(host(out), oracle.q8_gemv(xq, xs, wq, ws), "v7d_q8 n = 65536")
    x = rng.normal(0, 2, (2, n)).astype(F)
    v7g.q8_fused_gemv(out, dev(x), dev(wq), dev(ws))
    with np.errstate(all="ignore"):
        assert_same_f32(host(out), oracle.q8_fused_gemv(x, wq, ws), "v7d_q8_fused n = 65536")
    gq, gs = ref_fill(rng, (d, n), np.int8), ref_fill(rng, (d, n // 64), F)
    uq, us = ref_fill(rng, (d, n), np.int8), ref_fill(rng, (d, n // 64), F)
    xq1, xs1 = ref_fill(rng, (2, n), np.int8), ref_fill(rng, (2, n // 64), F)
    v7g.swiglu_q8_gemv(out, dev(xq1), dev(xs1), dev(gq), dev(gs), dev(uq), dev(us))
    with np.errstate(all="ignore"):
        assert_same_f32(host(out), oracle.swiglu_q8_gemv(xq1, xs1, gq, gs, uq, us), "v7d_swiglu_q8 n = 65536")
    xf = ref_fill(rng, (2, n), F)
    v7g.swiglu_f32q8_gemv(out, dev(xf), dev(gq), dev(gs), dev(uq), dev(us))
    with np.errstate(all="ignore"):
        assert_same_f32(host(out), oracle.swiglu_f32q8_gemv(xf, gq, gs, uq, us), "v7d_swiglu n = 65536")
    m = n + 64
    with pytest.raises(v7g.V7GError, match="at most 65536"):
        v7g.q8_gemv(torch.empty(1, 4, device=cuda), torch.zeros(1, m, dtype=torch.int8, device=cuda),
                    torch.zeros(1, m // 64, device=cuda), torch.zeros(4, m, dtype=torch.int8, device=cuda),
                    torch.zeros(4, m // 64, device=cuda))


@pytest.mark.parametrize("n,d", [(8192, 2048), (1024, 3000)])
@pytest.mark.parametrize("batch", [2, 4, 5, 9])
def test_gemv_token_blocks(cuda, oracle, n, d, batch):
    """A batch of two or more activation rows takes the streaming kernel's
    token blocks (two or four rows a CTA sharing one weight stream, the last
    block possibly partial): every row equal to the oracle's one-row product,
    with -128 weight bytes in some groups (the correction path of a block)."""
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(n + d + 31 * batch)
    xq, xs, gq, gs = q8_case(rng, batch, n, d)
    _, _, uq, us = q8_case(rng, 1, n, d)
    gq[::5, 3::97] = -128
    out = torch.empty(batch, d, device=cuda)
    v7g.q8_gemv(out, dev(xq), dev(xs), dev(gq), dev(gs))
    assert_same_f32(host(out), oracle.q8_gemv(xq, xs, gq, gs), f"v7d_q8 batch {batch}")
    out2 = torch.empty(batch, d, device=cuda)
    v7g.swiglu_q8_gemv(out2, dev(xq), dev(xs), dev(gq), dev(gs), dev(uq), dev(us))
    with np.errstate(all="ignore"):
        assert_same_f32(host(out2), oracle.swiglu_q8_gemv(xq, xs, gq, gs, uq, us), f"v7d_swiglu_q8 batch {batch}")


def test_gemv_token_blocks_long_rows(cuda, oracle):
    """Rows long enough (n = 32768) that four staged activations do not fit
    beside the weight stages: the call steps down to blocks of two rows (or
    one, or the fallback kernels), with every row equal to the oracle."""
    import v7multiplikator_b200 as v7g
    batch, n, d = 5, 32768, 64
    rng = np.random.default_rng(32768)
    xq, xs, gq, gs = q8_case(rng, batch, n, d)
    _, _, uq, us = q8_case(rng, 1, n, d)
    out = torch.empty(batch, d, device=cuda)
    v7g.q8_gemv(out, dev(xq), dev(xs), dev(gq), dev(gs))
    assert_same_f32(host(out), oracle.q8_gemv(xq, xs, gq, gs), "v7d_q8 n = 32768")
    v7g.swiglu_q8_gemv(out, dev(xq), dev(xs), dev(gq), dev(gs), dev(uq), dev(us))
    with np.errstate(all="ignore"):
        assert_same_f32(host(out), oracle.swiglu_q8_gemv(xq, xs, gq, gs, uq, us), "v7d_swiglu_q8 n = 32768")


def test_gemv_token_blocks_many(cuda, oracle):
    """Many token blocks (4099 rows: 1025 blocks of four, the last with
    three) through the streaming kernel, against the oracle."""
    import v7multiplikator_b200 as v7g
    batch, n, d = 4099, 256, 40
    rng = np.random.default_rng(11)
    xq, xs, wq, ws = q8_case(rng, batch, n, d)
    out = torch.empty(batch, d, device=cuda)
    v7g.q8_gemv(out, dev(xq), dev(xs), dev(wq), dev(ws))
    assert_same_f32(host(out), oracle.q8_gemv(xq, xs, wq, ws), "v7d_q8 batch 4099")


def test_gemv_largest_batch(cuda, oracle):
    """The largest batch (65535 activation rows: the grid's second dimension)
    against the oracle; one row more is refused."""
    import v7multiplikator_b200 as v7g
    batch, n, d = 65535, 64, 8
    rng = np.random.default_rng(7)
    xq, xs, wq, ws = q8_case(rng, batch, n, d)
    out = torch.empty(batch, d, device=cuda)
    v7g.q8_gemv(out, dev(xq), dev(xs), dev(wq), dev(ws))
    assert_same_f32(host(out), oracle.q8_gemv(xq, xs, wq, ws), "v7d_q8 batch 65535")
    with pytest.raises(v7g.V7GError, match="above 65535"):
        v7g.q8_gemv(torch.empty(batch + 1, d, device=cuda), torch.zeros(batch + 1, n, dtype=torch.int8, device=cuda),
                    torch.zeros(batch + 1, 1, device=cuda), dev(wq), dev(ws))
