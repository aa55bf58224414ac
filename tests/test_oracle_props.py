"""Properties of the oracle that the reference's C references do not pin:
the polynomial sigmoid against double-precision exp, the position-dependent
NaN behaviour of the Q8 group maximum (checked against an independent Python
restatement of the MAXPS tree), chain equalities the reference guarantees
(SwiGLU+Q8 = quantize(SwiGLU), RMSNorm+Q8 = quantize(RMSNorm)), and float64
sanity bounds for the norms."""
from __future__ import annotations

import numpy as np
import pytest

F = np.float32
FLOOR = F(1.4928778e-36)


def x86_max(a, b):
    return a if a > b else b


def py_group_absmax(x: np.ndarray) -> np.float32:
    """quantize_kernel.inc:62-84, restated without the C oracle."""
    a = [F(abs(v)) for v in x]
    m = []
    for c in range(8):
        m01 = x86_max(a[c], a[8 + c])
        m23 = x86_max(a[16 + c], a[24 + c])
        m45 = x86_max(a[32 + c], a[40 + c])
        m67 = x86_max(a[48 + c], a[56 + c])
        m.append(x86_max(x86_max(m01, m23), x86_max(m45, m67)))
    v = [x86_max(m[j], m[j + 4]) for j in range(4)]
    w = x86_max(x86_max(v[0], v[2]), x86_max(v[1], v[3]))
    return x86_max(w, FLOOR)


def py_code(p: np.float32) -> int:
    if not (abs(p) < 2147483648.0):
        return -127
    q = int(np.rint(p))
    return max(-127, min(127, q))


def py_quantize_group(x: np.ndarray):
    wmax = py_group_absmax(x)
    with np.errstate(all="ignore"):
        scale = F(wmax) / F(127.0)
        recip = F(1.0) / scale
        codes = [py_code(F(v) * recip) for v in x]
    return np.array(codes, np.int8), scale


def same_float(a, b):
    return (np.isnan(a) and np.isnan(b)) or a == b


@pytest.mark.parametrize("special", [np.nan, np.inf, -np.inf])
def test_group_max_position_semantics(oracle, special):
    rng = np.random.default_rng(7)
    for pos in range(64):
        x = rng.normal(0, 3, 64).astype(F)
        x[pos] = special
        q, s = oracle.quantize(x[None])
        eq, es = py_quantize_group(x)
        assert same_float(s[0, 0], es), (pos, s[0, 0], es)
        np.testing.assert_array_equal(q[0], eq, err_msg=f"position {pos}")


def test_group_two_nans(oracle):
    rng = np.random.default_rng(8)
    for trial in range(200):
        x = rng.normal(0, 1, 64).astype(F)
        i, j = rng.choice(64, 2, replace=False)
        x[i] = np.nan
        x[j] = np.nan if trial % 2 else np.inf
        q, s = oracle.quantize(x[None])
        eq, es = py_quantize_group(x)
        assert same_float(s[0, 0], es)
        np.testing.assert_array_equal(q[0], eq)


def test_tail_group_ignores_nan(oracle):
    """A trailing group (< 64 elements) folds MAXSS(|x_i|, wmax), which drops NaN
    (quantize_kernel.inc:125-131), and clamps before converting (:143-148)."""
    x = np.linspace(-5, 5, 100).astype(F)
    x[70] = np.nan
    q, s = oracle.quantize(x[None])
    tail = x[64:]
    wmax = max(F(abs(v)) for v in tail if not np.isnan(v))
    scale = F(wmax) / F(127)
    assert s[0, 1] == scale
    recip = F(1) / scale
    for k, v in enumerate(tail):
        p = F(v) * recip
        p = F(-127) if not (p > -127) else p
        p = p if p < 127 else F(127)
        assert q[0, 64 + k] == int(np.rint(p))


def test_all_zero_group_scale_is_flt_min(oracle):
    q, s = oracle.quantize(np.zeros((3, 128), F))
    assert np.all(q == 0)
    assert np.all(s == np.finfo(F).tiny)


def test_denormals_flush_in_quantize(oracle):
    """The quantiser runs with FTZ+DAZ (utility_dispatch.inc:127): subnormal
    inputs read as zero."""
    x = np.full((1, 64), 1e-39, F)
    q, s = oracle.quantize(x)
    assert np.all(q == 0) and s[0, 0] == np.finfo(F).tiny


def test_sigmoid_accuracy(oracle):
    g = np.concatenate([np.linspace(-100, 100, 20001), [0.0, -0.0, 80.0, -80.0, 79.99, 1e-30]]).astype(F)
    got = np.array([oracle.sigmoid(float(v)) for v in g], np.float64)
    t = np.clip(-g.astype(np.float64), -80, 80)
    ref = 1.0 / (1.0 + np.exp(t))
    rel = np.abs(got - ref) / ref
    # polynomial max rel err 1.27e-7 (v7_macros.inc:129-131) plus the error
    # of fx = -g*log2e in fp32: half an ulp of fx and the 1.3e-8 relative error
    # of log2e rounded to fp32, which become a relative error of ln2 * |dfx| in
    # 2^fx -- up to ~4e-6 near |g| = 80.  Inherent to the reference's method.
    fx = np.abs(t * np.log2(np.e)).astype(F).astype(np.float64)
    bound = 3e-7 + np.log(2) * (0.5 * np.spacing(fx.astype(F)).astype(np.float64) + 1.4e-8 * fx)
    assert np.all(rel <= bound)


def test_sigmoid_nan_clamps(oracle):
    # MAXPS(-NaN, -80) returns -80: sigmoid(NaN) = 1 / (1 + 2^-115.4...)
    assert oracle.sigmoid(float("nan")) == oracle.sigmoid(80.0)


def test_swiglu_q8_equals_quantize_of_swiglu(oracle):
    rng = np.random.default_rng(1)
    g = rng.normal(0, 2, (33, 192)).astype(F)
    u = rng.normal(0, 2, (33, 192)).astype(F)
    q, s = oracle.swiglu_q8(g, u)
    q2, s2 = oracle.quantize(oracle.swiglu(g, u))
    np.testing.assert_array_equal(q, q2)
    np.testing.assert_array_equal(s, s2)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_swiglu_q8_avx2_equals_scalar(oracle, seed):
    """The AVX2 form of SwiGLU -> Q8 (the one the CPU baseline times) gives
    the scalar restatement's bits: ordinary N(0, 2) rows, and rows planted
    with NaN, infinities, subnormals, huge values, signed zeros, all-zero and
    all-subnormal groups (every position of the MAXPS tree gets a NaN)."""
    rng = np.random.default_rng(seed)
    rows, n = 67, 1024
    g = rng.normal(0, 2, (rows, n)).astype(np.float32)
    u = rng.normal(0, 2, (rows, n)).astype(np.float32)
    specials = np.array([np.nan, np.inf, -np.inf, 1e-40, -1e-42, 3e38, -3e38, 0.0, -0.0, 85.0, -85.0, 1e-30], np.float32)
    for arr in (g, u):
        flat = arr.reshape(-1)
        idx = rng.choice(flat.size, flat.size // 50, replace=False)
        flat[idx] = specials[rng.integers(0, specials.size, idx.size)]
    g[3, :64] = 0.0
    u[3, :64] = 0.0
    g[4, 64:128] = 1e-40
    for pos in range(64):  # a NaN at every position of a group, one group each (rows 5..8)
        g[5 + pos // 16, 64 * (pos % 16) + pos] = np.nan
    q_a, s_a = oracle.swiglu_q8_avx2(g, u)
    q_s, s_s = oracle.swiglu_q8(g, u)
    assert np.array_equal(q_a, q_s)
    assert np.array_equal(s_a.view(np.uint32), s_s.view(np.uint32))


def test_swiglu_vs_float64(oracle):
    rng = np.random.default_rng(2)
    g = rng.normal(0, 2, 100000).astype(F)
    u = rng.normal(0, 2, 100000).astype(F)
    out = oracle.swiglu(g, u).astype(np.float64)
    ref = g.astype(np.float64) / (1 + np.exp(-g.astype(np.float64))) * u
    assert np.all(np.abs(out - ref) <= 1e-6 + 2e-6 * np.abs(ref))


def test_rmsnorm_quantize_equals_chain(oracle):
    """kt_verify_rmsnorm_quantize's guarantee (kt_utils.h:850-932): the fused
    kernel's codes equal rmsnorm -> quantize bit for bit."""
    rng = np.random.default_rng(3)
    for n in (64, 128, 1024, 2048, 3072, 8192):
        x = rng.uniform(-1, 1, (4, n)).astype(F)
        w = rng.uniform(0.5, 1.5, n).astype(F)
        q, s = oracle.rmsnorm_quantize(x, w, 1e-6)
        q2, s2 = oracle.quantize(oracle.rmsnorm(x, w, 1e-6))
        np.testing.assert_array_equal(q, q2)
        np.testing.assert_array_equal(s, s2)


@pytest.mark.parametrize("n", [32, 64, 96, 2048, 4096])
def test_rmsnorm_vs_float64(oracle, n):
    rng = np.random.default_rng(n)
    x = rng.normal(0, 1, (16, n)).astype(F)
    w = rng.normal(1, 0.1, n).astype(F)
    out = oracle.rmsnorm(x, w, 1e-6).astype(np.float64)
    xd = x.astype(np.float64)
    ref = xd / np.sqrt((xd * xd).mean(1, keepdims=True) + 1e-6) * w
    assert np.all(np.abs(out - ref) <= 1e-6 + 1e-5 * np.abs(ref))


@pytest.mark.parametrize("n", [8, 16, 24, 40, 48, 2048])
def test_fused_add_rmsnorm_vs_float64(oracle, n):
    rng = np.random.default_rng(n)
    r = rng.normal(0, 1, (8, n)).astype(F)
    a = rng.normal(0, 0.5, (8, n)).astype(F)
    w = rng.normal(1, 0.1, n).astype(F)
    out, res = oracle.fused_add_rmsnorm(r, a, w, 1e-6)
    np.testing.assert_array_equal(res, r + a)
    sd = res.astype(np.float64)
    ref = sd / np.sqrt((sd * sd).mean(1, keepdims=True) + 1e-6) * w
    assert np.all(np.abs(out - ref) <= 1e-6 + 1e-5 * np.abs(ref))


def test_rope_vs_float64(oracle):
    rng = np.random.default_rng(4)
    T, H, D = 9, 3, 128
    x = rng.normal(0, 1, (T, H, D)).astype(F)
    w = rng.normal(1, 0.1, D).astype(F)
    cos, sin = oracle.rope_tables(T + 5, D // 2, D // 2, 1e6)
    pos0 = 5
    out = oracle.rope(x, w, cos, sin, pos0, 1e-6).astype(np.float64)
    xd = x.astype(np.float64)
    nrm = xd / np.sqrt((xd * xd).mean(-1, keepdims=True) + 1e-6) * w
    c = cos[pos0:pos0 + T, None, :].astype(np.float64)
    s = sin[pos0:pos0 + T, None, :].astype(np.float64)
    e, o = nrm[..., :D // 2], nrm[..., D // 2:]
    ref = np.concatenate([e * c - o * s, e * s + o * c], -1)
    assert np.all(np.abs(out - ref) <= 1e-6 + 1e-5 * np.abs(ref))


def test_rope_position_zero_only_normalises(oracle):
    rng = np.random.default_rng(5)
    x = rng.normal(0, 1, (1, 4, 64)).astype(F)
    w = rng.normal(1, 0.1, 64).astype(F)
    cos = np.full((1, 32), 0.3, F)  # would rotate if it were applied
    sin = np.full((1, 32), 0.9, F)
    out = oracle.rope(x, w, cos, sin, 0, 1e-6)
    xd = x.astype(np.float64)
    ref = xd / np.sqrt((xd * xd).mean(-1, keepdims=True) + 1e-6) * w
    assert np.all(np.abs(out - ref) <= 1e-6 + 1e-5 * np.abs(ref))


def test_contract_violations(oracle):
    with pytest.raises(ValueError):
        oracle.rmsnorm(np.zeros((1, 48), F), np.zeros(48, F), 1e-6)  # 48 % 32 != 0
    with pytest.raises(ValueError):
        oracle.fused_add_rmsnorm(np.zeros((1, 12), F), np.zeros((1, 12), F), np.zeros(12, F), 1e-6)
    with pytest.raises(ValueError):
        oracle.swiglu_q8(np.zeros((1, 96), F), np.zeros((1, 96), F))


def test_thread_count_invariance(oracle):
    from oracle.pyoracle import Oracle
    one = Oracle(nthreads=1)
    rng = np.random.default_rng(6)
    g = rng.normal(0, 2, (37, 256)).astype(F)
    u = rng.normal(0, 2, (37, 256)).astype(F)
    a = oracle.swiglu_q8(g, u)
    b = one.swiglu_q8(g, u)
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1], b[1])
