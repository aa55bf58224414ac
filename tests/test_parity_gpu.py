"""Parity of the sm_100a kernels with the oracle, called through the C-ABI.

The kernels reproduce the reference's arithmetic operation for operation, so
the bar here is bit-exactness: fp32 outputs equal the oracle's bit for bit
(NaN compared as NaN, since x86 and the GPU encode NaN payloads differently),
Q8 codes and scales equal exactly.  The BASELINE tolerance (|d| <= 1e-6 +
1e-5 |ref| for fp32; Q8 codes exact except +-1 at exact ties; scales within 1
ulp) is therefore met with margin; it is asserted separately against float64
where the oracle is not the reference.  Inputs: seeded N(0, sigma) draws, the
reference validators' own fills, and planted specials (NaN, inf, zeros,
subnormals) at every position that matters.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import reffills as rf

pytestmark = pytest.mark.gpu
F = np.float32


def dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t: torch.Tensor) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy()


def assert_same_f32(got: np.ndarray, want: np.ndarray, msg: str = "") -> None:
    got = np.asarray(got, F)
    want = np.asarray(want, F)
    assert got.shape == want.shape, msg
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan), f"NaN positions differ {msg}"
    g, w = got[~nan].view(np.uint32), want[~nan].view(np.uint32)
    bad = np.nonzero(g != w)[0]
    assert bad.size == 0, f"{bad.size} mismatches {msg}: first at {bad[0]}: got {got[~nan][bad[0]]!r} want {want[~nan][bad[0]]!r}"


def normal(rng, shape, mean=0.0, std=1.0):
    return rng.normal(mean, std, shape).astype(F)


# ------------------------------------------------- the fast arithmetic itself


def test_selftest_arith_exhaustive(cuda):
    """The Markstein reciprocal / divide and the packed SiLU and Q8 code paths
    equal the IEEE instructions on every input they can receive (2^23
    mantissas x every exponent, all 2^32 patterns for the SiLU and codes), and
    the Q8 code paths round the product h * recip before rounding it to a code
    (2^31 products within a few ulps of a tie, non-trivial reciprocals)."""
    import v7multiplikator_b200 as v7g
    assert v7g.selftest_arith() == [0, 0, 0, 0, 0, 0, 0]


# --------------------------------------------------------------- RMSNorm rows



def rope_tables_for(oracle, rng, rows, half, rmd, base):
    """cos/sin tables [rows, rmd]: the reference's own builder (x87, through the
    oracle) up to the 256 frequency pairs it makes; beyond that -- head_dim up to
    1024, which the kernels take with caller tables -- seeded unit-circle values."""
    if half <= 256:
        return oracle.rope_tables(rows, half, rmd, base)
    th = rng.uniform(-np.pi, np.pi, (rows, rmd))
    return np.cos(th).astype(np.float32), np.sin(th).astype(np.float32)

@pytest.mark.parametrize("rows,n", [(1, 32), (3, 64), (17, 96), (64, 2048), (5, 3072), (2, 8192), (7, 4096), (300, 256),
                                    (1025, 96), (2000, 2048), (257, 32), (777, 4096), (400, 8192), (600, 13000 // 32 * 32)])
@pytest.mark.parametrize("eps", [0.0, 1e-6])
def test_rmsnorm_rows(cuda, oracle, rows, n, eps):
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(rows * 131 + n)
    x = normal(rng, (rows, n))
    w = normal(rng, n, 1.0, 0.1)
    out = torch.empty(rows, n, device=cuda)
    v7g.rmsnorm_rows(out, dev(x), dev(w), eps)
    assert_same_f32(host(out), oracle.rmsnorm(x, w, eps))


def test_rmsnorm_in_place_and_specials(cuda, oracle):
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(3)
    x = normal(rng, (6, 128))
    x[1, 5] = np.inf
    x[2, 100] = np.nan
    x[3] = 0.0
    x[4] = 1e-39  # subnormal: no FTZ in the direct-call kernels
    x[5, ::3] = -0.0
    w = normal(rng, 128, 1.0, 0.1)
    t = dev(x)
    with np.errstate(all="ignore"):
        want = oracle.rmsnorm(x, w, 1e-6)
    v7g.rmsnorm_rows(t, t, dev(w), 1e-6)
    assert_same_f32(host(t), want)


@pytest.mark.parametrize("size", [64, 128, 256, 1024, 2048, 3072, 8192])
@pytest.mark.parametrize("seed", [12345, 67890])
def test_rmsnorm_reference_validator_cases(cuda, oracle, golden, size, seed):
    """v_rmsnorm_validate section 1 through the reference-named op: within the
    validator's 1e-3 of its C reference, bit-exact against the oracle."""
    import v7multiplikator_b200 as v7g
    x, w = rf.rmsnorm_case(size, seed)
    v7g.set_rms_eps(1e-6)
    o = torch.empty(size, device=cuda)
    v7g.v7s_rmsnorm(o, dev(x), dev(w))
    got = host(o)
    assert np.max(np.abs(got - golden[f"rmsnorm/{size}/{seed}"])) <= 1e-3
    assert_same_f32(got, oracle.rmsnorm(x[None], w, 1e-6)[0])


# --------------------------------------------------- fused add + RMSNorm rows


def test_row_kernels_in_place_at_pipeline_sizes(cuda, oracle):
    """Hundreds of rows (the shared-memory row pipeline): RMSNorm with the
    output over its input, and fused add + RMSNorm with the output over the
    residual (the output is the last write, as in the reference)."""
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(17)
    x = normal(rng, (600, 2048))
    w = normal(rng, 2048, 1.0, 0.1)
    t = dev(x)
    v7g.rmsnorm_rows(t, t, dev(w), 1e-6)
    assert_same_f32(host(t), oracle.rmsnorm(x, w, 1e-6))
    r = normal(rng, (600, 2048))
    a = normal(rng, (600, 2048), 0, 0.5)
    rt = dev(r)
    v7g.fused_add_rmsnorm_rows(rt, rt, dev(a), dev(w), 1e-6)
    want_o, _ = oracle.fused_add_rmsnorm(r, a, w, 1e-6)
    assert_same_f32(host(rt), want_o, "out over residual")


@pytest.mark.parametrize("rows,n", [(1, 8), (3, 16), (2, 24), (5, 48), (4, 64), (33, 2048), (3, 3072), (2, 8192), (9, 40),
                                    (1025, 40), (2000, 2048), (513, 8), (300, 24), (700, 2056), (400, 4096), (260, 12296)])
def test_fused_add_rmsnorm_rows(cuda, oracle, rows, n):
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(rows * 7 + n)
    r = normal(rng, (rows, n))
    a = normal(rng, (rows, n), 0, 0.5)
    w = normal(rng, n, 1, 0.1)
    rt, out = dev(r), torch.empty(rows, n, device=cuda)
    v7g.fused_add_rmsnorm_rows(out, rt, dev(a), dev(w), 1e-6)
    want_o, want_r = oracle.fused_add_rmsnorm(r, a, w, 1e-6)
    assert_same_f32(host(rt), want_r, "residual")
    assert_same_f32(host(out), want_o, "out")


@pytest.mark.parametrize("dim", [8, 16, 24, 48, 64, 128, 256, 1024, 2048, 3072, 8192])
def test_fused_add_rmsnorm_reference_validator_cases(cuda, oracle, golden, dim):
    import v7multiplikator_b200 as v7g
    for seed in (12345, 67890):
        r, a, w = rf.add_rmsnorm_case(dim, seed)
        v7g.set_rms_eps(1e-6)
        o, rt = torch.empty(dim, device=cuda), dev(r)
        v7g.v7s_fused_add_rmsnorm(o, rt, dev(a), dev(w))
        got = host(o)
        assert np.max(np.abs(got - golden[f"add_rmsnorm/{dim}/{seed}"])) <= 1e-3
        assert np.array_equal(host(rt), golden[f"add_rmsnorm_res/{dim}/{seed}"])
        want_o, _ = oracle.fused_add_rmsnorm(r[None], a[None], w, 1e-6)
        assert_same_f32(got, want_o[0])


# ------------------------------------------------------------ RMSNorm + RoPE


@pytest.mark.parametrize("head_dim", [32, 64, 96, 128, 192, 256, 512, 1024])
@pytest.mark.parametrize("heads", [(16, 8), (5, 3), (0, 2), (4, 0)])
@pytest.mark.parametrize("tokens,pos0", [(1, 0), (7, 0), (130, 5)])
def test_rmsnorm_rope_rows(cuda, oracle, head_dim, heads, tokens, pos0):
    import v7multiplikator_b200 as v7g
    hq, hk = heads
    rng = np.random.default_rng(head_dim * 1000 + hq * 10 + hk + tokens)
    q = normal(rng, (tokens, hq, head_dim))
    k = normal(rng, (tokens, hk, head_dim))
    wq = normal(rng, head_dim, 1, 0.1)
    wk = normal(rng, head_dim, 1, 0.1)
    rmd = head_dim  # validator layout: rows of head_dim, first half used
    cos, sin = rope_tables_for(oracle, rng, pos0 + tokens, head_dim // 2, rmd, 1e6)
    qt, kt = dev(q), dev(k)
    v7g.rmsnorm_rope_rows(qt if hq else None, kt if hk else None, dev(wq) if hq else None, dev(wk) if hk else None,
                          dev(cos), dev(sin), pos0, 1e-6)
    if hq:
        assert_same_f32(host(qt), oracle.rope(q, wq, cos, sin, pos0, 1e-6), "q")
    if hk:
        assert_same_f32(host(kt), oracle.rope(k, wk, cos, sin, pos0, 1e-6), "k")


@pytest.mark.parametrize("case", [(1, 64, 0, 64, 1e-6), (1, 64, 7, 64, 1e-6), (4, 64, 31, 64, 1e-6), (8, 128, 0, 128, 1e-6),
                                  (40, 64, 31, 64, 1e-6), (40, 128, 7, 128, 1e-6), (32, 64, 31, 64, 1e-5)])
def test_rope_reference_validator_cases(cuda, oracle, golden, case):
    import v7multiplikator_b200 as v7g
    h, d, pos, rmd, eps = case
    for seed in (12345, 67890):
        key = f"{h}x{d}/{pos}/{rmd}/{'1e-5' if eps == 1e-5 else '1e-6'}/{seed}"
        buf, w = rf.rope_case(h, d, seed)
        cos, sin = golden[f"rope_cos/{key}"], golden[f"rope_sin/{key}"]
        v7g.set_rms_eps(eps)
        bt = dev(buf)
        v7g.v7s_rmsnorm_rope_heads(bt, h, d, dev(w), dev(cos), dev(sin), pos, rmd)
        got = host(bt)
        assert np.max(np.abs(got - golden[f"rope/{key}"])) <= 1e-3
        assert_same_f32(got, oracle.rope(buf.reshape(1, h, d), w, cos, sin, pos, eps, rope_max_dim=rmd).reshape(-1))
    v7g.set_rms_eps(1e-6)


# ------------------------------------------------------------------- SwiGLU


SPECIALS = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 80.0, -80.0, 81.0, -81.0, 1e-39, -1e-39, 3e38, -3e38, 1e-30], F)


@pytest.mark.parametrize("count", [1, 3, 4, 1000, 4097, 1 << 20])
def test_swiglu(cuda, oracle, count):
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(count)
    g = normal(rng, count, 0, 2)
    u = normal(rng, count, 0, 2)
    if count >= 1000:
        g[:SPECIALS.size] = SPECIALS
        u[SPECIALS.size:2 * SPECIALS.size] = SPECIALS
    out = torch.empty(count, device=cuda)
    v7g.swiglu(out, dev(g), dev(u))
    with np.errstate(all="ignore"):
        assert_same_f32(host(out), oracle.swiglu(g, u))


def test_swiglu_unaligned(cuda, oracle):
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(11)
    g = normal(rng, 1001, 0, 2)
    u = normal(rng, 1001, 0, 2)
    gt, ut = dev(g), dev(u)
    out = torch.empty(1001, device=cuda)
    v7g.swiglu(out[1:], gt[1:], ut[1:])  # 4-byte offset: the scalar kernel
    assert_same_f32(host(out)[1:], oracle.swiglu(g[1:], u[1:]))


def test_swiglu_vs_float64(cuda):
    """BASELINE tolerance against float64 SiLU: the polynomial sigmoid is within
    1e-6 abs + 1e-5 rel of the exact one for N(0, 2) inputs."""
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(12)
    g = normal(rng, 1 << 20, 0, 2)
    u = normal(rng, 1 << 20, 0, 2)
    out = torch.empty(1 << 20, device=cuda)
    v7g.swiglu(out, dev(g), dev(u))
    gd, ud = g.astype(np.float64), u.astype(np.float64)
    ref = gd / (1 + np.exp(-gd)) * ud
    assert np.all(np.abs(host(out) - ref) <= 1e-6 + 1e-5 * np.abs(ref))


# --------------------------------------------------------------- Q8 kernels


def plant(x: np.ndarray, rng, count: int) -> np.ndarray:
    flat = x.reshape(-1)
    idx = rng.choice(flat.size, count, replace=False)
    flat[idx] = rng.choice(np.array([np.nan, np.inf, -np.inf, 0.0, 1e-39, 1e30], F), count)
    return x


@pytest.mark.parametrize("rows,n", [(1, 64), (3, 128), (5, 192), (33, 12288), (2, 448), (1, 64 * 1001), (1, 1 << 22)])
@pytest.mark.parametrize("specials", [False, True])
def test_swiglu_q8_rows(cuda, oracle, rows, n, specials):
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(rows * n + specials)
    g = normal(rng, (rows, n), 0, 2)
    u = normal(rng, (rows, n), 0, 2)
    if specials:
        plant(g, rng, max(1, g.size // 500))
        plant(u, rng, max(1, u.size // 500))
    codes = torch.empty(rows, n, dtype=torch.int8, device=cuda)
    scales = torch.empty(rows, n // 64, device=cuda)
    v7g.swiglu_q8_rows(codes, scales, dev(g), dev(u))
    with np.errstate(all="ignore"):
        wq, ws = oracle.swiglu_q8(g, u)
    np.testing.assert_array_equal(host(codes), wq)
    assert_same_f32(host(scales), ws)


def test_swiglu_q8_general_kernel(cuda, oracle):
    """Unaligned operands take the one-warp-per-group kernel: same results."""
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(21)
    g = normal(rng, (4 * 256 + 1,), 0, 2)
    u = normal(rng, (4 * 256 + 1,), 0, 2)
    gt, ut = dev(g), dev(u)
    codes = torch.empty(4 * 256 + 1, dtype=torch.int8, device=cuda)
    scales = torch.empty(16, device=cuda)
    v7g.swiglu_q8_rows(codes[1:].view(4, 256), scales, gt[1:].view(4, 256), ut[1:].view(4, 256))
    wq, ws = oracle.swiglu_q8(g[1:].reshape(4, 256), u[1:].reshape(4, 256))
    np.testing.assert_array_equal(host(codes)[1:].reshape(4, 256), wq)
    assert_same_f32(host(scales).reshape(4, 4), ws)


@pytest.mark.parametrize("rows,n", [(1, 1), (1, 63), (1, 64), (7, 100), (3, 4096), (1, 65536), (5, 12288), (2, 130)])
@pytest.mark.parametrize("specials", [False, True])
def test_quantize_rows(cuda, oracle, rows, n, specials):
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(rows * n + 7 * specials)
    x = normal(rng, (rows, n), 0, 3)
    if specials:
        plant(x, rng, max(1, x.size // 100))
    ng = (n + 63) // 64
    codes = torch.empty(rows, n, dtype=torch.int8, device=cuda)
    scales = torch.empty(rows, ng, device=cuda)
    v7g.quantize_rows(codes, scales, dev(x))
    with np.errstate(all="ignore"):
        wq, ws = oracle.quantize(x)
    np.testing.assert_array_equal(host(codes), wq)
    assert_same_f32(host(scales), ws)


def test_quantize_nan_at_every_position(cuda, oracle):
    """The NaN behaviour of the MAXPS tree depends on where the NaN sits; both
    kernel layouts (half-warp float4 and warp-per-group) must follow it."""
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(31)
    x = normal(rng, (128, 64), 0, 2)
    for p in range(64):
        x[p, p] = np.nan
        x[64 + p, p] = np.nan
        x[64 + p, (p * 7 + 3) % 64] = np.inf
    with np.errstate(all="ignore"):
        wq, ws = oracle.quantize(x)
    for offset in (0, 1):  # aligned: flat kernel; offset: general kernel
        buf = torch.zeros(128 * 64 + 1, device=cuda)
        buf[offset:offset + 128 * 64] = dev(x).view(-1)
        cbuf = torch.zeros(128 * 64 + 1, dtype=torch.int8, device=cuda)
        codes = cbuf[offset:offset + 128 * 64].view(128, 64)
        scales = torch.empty(128, 1, device=cuda)
        v7g.quantize_rows(codes, scales, buf[offset:offset + 128 * 64].view(128, 64))
        np.testing.assert_array_equal(host(codes), wq)
        assert_same_f32(host(scales), ws)


@pytest.mark.parametrize("pattern", range(7), ids=rf.QUANT_PATTERNS)
def test_quantize_reference_validator_cases(cuda, golden, pattern):
    """v_quantize_validate through the reference-named op: codes bit-exact
    against the reference's C reference (kt_utils.h:703-730)."""
    import hashlib
    import v7multiplikator_b200 as v7g
    for n in (64, 256, 1024, 4096, 8192, 65536):
        for seed in (12345, 67890, 11111):
            x = rf.quantize_pattern(n, seed, pattern)
            q = torch.empty(n, dtype=torch.int8, device=cuda)
            s = torch.empty((n + 63) // 64, device=cuda)
            v7g.v7d_quantize(q, dev(x), s)
            key = f"{pattern}/{n}/{seed}"
            assert hashlib.sha256(host(q).tobytes()).hexdigest() == bytes(golden[f"quant_codes_sha256/{key}"]).decode()


@pytest.mark.parametrize("rows,n", [(1, 64), (3, 128), (9, 2048), (2, 3072), (2, 8192), (1, 12288),
                                    (3000, 2048), (1500, 4096), (700, 64), (300, 8192), (257, 192), (500, 12288)])
def test_rmsnorm_quantize_rows(cuda, oracle, rows, n):
    """Up to 3000 rows: codes next to a rounding tie occur a few times per
    million elements, so small row counts alone would not show a product that
    lost its rounding."""
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(rows + n)
    x = rng.uniform(-1, 1, (rows, n)).astype(F)
    w = rng.uniform(0.5, 1.5, n).astype(F)
    codes = torch.empty(rows, n, dtype=torch.int8, device=cuda)
    scales = torch.empty(rows, n // 64, device=cuda)
    v7g.rmsnorm_quantize_rows(codes, scales, dev(x), dev(w), 1e-6)
    wq, ws = oracle.rmsnorm_quantize(x, w, 1e-6)
    np.testing.assert_array_equal(host(codes), wq)
    assert_same_f32(host(scales), ws)
    # the reference's guarantee: equal to rmsnorm -> quantize (kt_utils.h:850-932)
    xb = torch.empty(rows, n, device=cuda)
    v7g.rmsnorm_rows(xb, dev(x), dev(w), 1e-6)
    c2 = torch.empty_like(codes)
    s2 = torch.empty_like(scales)
    v7g.quantize_rows(c2, s2, xb)
    np.testing.assert_array_equal(host(c2), host(codes))


def test_rmsnorm_quantize_specials_at_every_group_position(cuda, oracle):
    """NaN and infinities in gamma at each of a group's 64 positions (and in
    every group slot of a warp): the absmax must follow the reference's MAXPS
    tree order, which decides which NaN survives."""
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(77)
    rows, n = 3, 256
    x = rng.uniform(-1, 1, (rows, n)).astype(F)
    codes = torch.empty(rows, n, dtype=torch.int8, device=cuda)
    scales = torch.empty(rows, n // 64, device=cuda)
    for p in range(64):
        w = rng.uniform(0.5, 1.5, n).astype(F)
        w[p] = np.nan                      # group 0
        w[64 + (p * 7) % 64] = -np.inf     # group 1
        w[128 + p] = np.inf                # group 2
        w[128 + (p + 32) % 64] = np.nan
        w[192 + (p * 5) % 64] = 1e-39      # group 3: subnormal gamma (DAZ)
        v7g.rmsnorm_quantize_rows(codes, scales, dev(x), dev(w), 1e-6)
        with np.errstate(all="ignore"):
            wq, ws = oracle.rmsnorm_quantize(x, w, 1e-6)
        np.testing.assert_array_equal(host(codes), wq, err_msg=f"position {p}")
        assert_same_f32(host(scales), ws, f"position {p}")


@pytest.mark.parametrize("eps", [0.0, 1e-6])
def test_rmsnorm_pipeline_special_rows(cuda, oracle, eps):
    """The RMSNorm row pipeline (600 rows) on rows with NaN, infinities, an
    overflowing sum of squares, all zeros, subnormals (no FTZ here) and a
    huge value, among ordinary rows."""
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(91)
    rows, n = 600, 2048
    x = normal(rng, (rows, n))
    x[1, 17] = np.nan
    x[2, 1000] = np.inf
    x[3, 5] = -np.inf
    x[4] = 0.0
    x[5] = rng.uniform(1e19, 3e19, n).astype(F)
    x[6] = 1e-39
    x[7, 3] = 3e38
    x[590:597] = x[1:8]
    w = normal(rng, n, 1.0, 0.1)
    out = torch.empty(rows, n, device=cuda)
    v7g.rmsnorm_rows(out, dev(x), dev(w), eps)
    with np.errstate(all="ignore"):
        want = oracle.rmsnorm(x, w, eps)
    assert_same_f32(host(out), want)


@pytest.mark.parametrize("rows", [9, 300, 1200])
@pytest.mark.parametrize("gamma", ["plain", "nan", "inf", "huge", "tiny"])
@pytest.mark.parametrize("eps", [0.0, 1e-6])
def test_rmsnorm_quantize_special_rows(cuda, oracle, rows, gamma, eps):
    """Rows that must leave the finite-row shortcut -- NaN or infinities in x,
    a sum of squares that overflows, an all-zero row (infinite scale when eps is
    0), subnormal and huge values -- mixed among ordinary rows in one launch,
    under gammas that are tame or not (NaN, infinity, |w| >= 1e30, subnormal):
    each row takes its own path (the shortcut or the general one) and every
    code and scale equals the oracle's.  300 and 1200 rows run the row
    pipeline, 9 the register-chunk kernel."""
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(rows * 31 + len(gamma))
    n = 2048
    x = rng.uniform(-1, 1, (rows, n)).astype(F)
    specials = {1: ("nan", 17), 2: ("inf", 1000), 3: ("-inf", 5), 4: ("zero", None), 5: ("overflow", None),
                6: ("subnormal", None), 7: ("huge", 3)}
    for r, (kind, col) in specials.items():
        if kind == "nan":
            x[r, col] = np.nan
        elif kind == "inf":
            x[r, col] = np.inf
        elif kind == "-inf":
            x[r, col] = -np.inf
        elif kind == "zero":
            x[r] = 0.0
        elif kind == "overflow":
            x[r] = rng.uniform(1e19, 3e19, n).astype(F)  # squares overflow float
        elif kind == "subnormal":
            x[r] = 1e-39
        else:
            x[r, col] = 3e38
    if rows > 100:  # the same rows again deep into the launch (other warps and SMs)
        x[rows - 8:rows - 1] = x[1:8]
    w = rng.uniform(0.5, 1.5, n).astype(F)
    if gamma == "nan":
        w[700] = np.nan
    elif gamma == "inf":
        w[64] = np.inf
    elif gamma == "huge":
        w[5] = 2e30
    elif gamma == "tiny":
        w[::7] = 1e-39
    codes = torch.empty(rows, n, dtype=torch.int8, device=cuda)
    scales = torch.empty(rows, n // 64, device=cuda)
    v7g.rmsnorm_quantize_rows(codes, scales, dev(x), dev(w), eps)
    with np.errstate(all="ignore"):
        wq, ws = oracle.rmsnorm_quantize(x, w, eps)
    np.testing.assert_array_equal(host(codes), wq)
    assert_same_f32(host(scales), ws)


def test_rmsnorm_quantize_rejects_unaligned_codes(cuda):
    import v7multiplikator_b200 as v7g
    x = torch.zeros(2, 64, device=cuda)
    buf = torch.zeros(2 * 64 + 4, dtype=torch.int8, device=cuda)
    with pytest.raises(v7g.V7GError, match="aligned"):
        v7g.rmsnorm_quantize_rows(buf[4:].view(2, 64), torch.empty(2, 1, device=cuda), x, torch.ones(64, device=cuda), 1e-6)


# -------------------------------------------------------------- add_inplace


@pytest.mark.parametrize("count", [32, 96, 160, 2048, 4099, 1 << 22])
def test_add_inplace(cuda, oracle, count):
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(count)
    x = normal(rng, count, 0, 10)
    y = normal(rng, count, 0, 10)
    xt = dev(x)
    v7g.add_inplace(xt, dev(y))
    assert_same_f32(host(xt), oracle.add_inplace(x, y))
    if count == 160:
        xt = dev(x)
        v7g.add_inplace(xt[1:], dev(y)[1:])  # unaligned
        want = oracle.add_inplace(x, y)
        want[0] = x[0]
        assert_same_f32(host(xt), want)


def test_add_inplace_reference_validator_cases(cuda, golden):
    import v7multiplikator_b200 as v7g
    for n in (32, 64, 96, 128, 160, 1024, 2048):
        for seed in (12345, 67890):
            x, y = rf.add_inplace_case(n, seed)
            xt = dev(x)
            v7g.v7s_add_inplace(xt, dev(y))
            np.testing.assert_array_equal(host(xt), golden[f"add_inplace/{n}/{seed}"])


# ----------------------------------------------------- runtime behaviour


def test_errors_raise_and_count(cuda):
    import v7multiplikator_b200 as v7g
    before = v7g.launch_count()
    x = torch.zeros(4, 48, device=cuda)
    with pytest.raises(v7g.V7GError, match="multiple of 32"):
        v7g.rmsnorm_rows(torch.empty_like(x), x, torch.ones(48, device=cuda), 1e-6)
    assert v7g.launch_count() == before  # nothing launched
    y = torch.zeros(4, 64, device=cuda)
    v7g.rmsnorm_rows(torch.empty_like(y), y, torch.ones(64, device=cuda), 1e-6)
    assert v7g.launch_count() == before + 1


def test_fill_normal_is_shard_independent(cuda):
    import v7multiplikator_b200 as v7g
    full = torch.empty(64, 1000, device=cuda)
    v7g.fill_normal(full, seed=5, mean=0.0, std=2.0)
    part = torch.empty(16, 1000, device=cuda)
    v7g.fill_normal(part, seed=5, mean=0.0, std=2.0, row0=32)
    assert torch.equal(full[32:48], part)
    s = full.double()
    assert abs(s.mean().item()) < 0.05 and abs(s.std().item() - 2.0) < 0.05


def test_nonzero_stream(cuda, oracle):
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(41)
    g = normal(rng, (8, 256), 0, 2)
    u = normal(rng, (8, 256), 0, 2)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        gt, ut = dev(g), dev(u)
        codes = torch.empty(8, 256, dtype=torch.int8, device=cuda)
        scales = torch.empty(8, 4, device=cuda)
        v7g.swiglu_q8_rows(codes, scales, gt, ut)
    s.synchronize()
    wq, ws = oracle.swiglu_q8(g, u)
    np.testing.assert_array_equal(codes.cpu().numpy(), wq)


@pytest.mark.parametrize("rows,n", [(2, 1 << 20), (1, (1 << 24) - 64)])
def test_row_kernels_longest_rows(cuda, oracle, rows, n):
    """The longest rows the row kernels take (n below 2^24: a 64 MB row, one
    warp streaming it in chunks) for RMSNorm, fused add + RMSNorm and
    RMSNorm -> Q8, against the oracle; n = 2^24 is refused."""
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(n + rows)
    x = normal(rng, (rows, n))
    a = normal(rng, (rows, n), 0, 0.5)
    w = normal(rng, n, 1.0, 0.1)
    out = torch.empty(rows, n, device=cuda)
    v7g.rmsnorm_rows(out, dev(x), dev(w), 1e-6)
    assert_same_f32(host(out), oracle.rmsnorm(x, w, 1e-6), "rmsnorm")
    rt = dev(x)
    v7g.fused_add_rmsnorm_rows(out, rt, dev(a), dev(w), 1e-6)
    want_o, want_r = oracle.fused_add_rmsnorm(x, a, w, 1e-6)
    assert_same_f32(host(rt), want_r, "residual")
    assert_same_f32(host(out), want_o, "fused out")
    del rt, out
    codes = torch.empty(rows, n, dtype=torch.int8, device=cuda)
    scales = torch.empty(rows, n // 64, device=cuda)
    v7g.rmsnorm_quantize_rows(codes, scales, dev(x), dev(w), 1e-6)
    wq, ws = oracle.rmsnorm_quantize(x, w, 1e-6)
    np.testing.assert_array_equal(host(codes), wq)
    assert_same_f32(host(scales), ws)
    if rows == 1:
        m = 1 << 24
        with pytest.raises(v7g.V7GError, match="2\\^24"):
            v7g.rmsnorm_rows(torch.empty(1, m, device=cuda), torch.zeros(1, m, device=cuda), torch.ones(m, device=cuda), 1e-6)
