"""The oracle's Q8-weight GEMVs (v7d_q8, v7d_q8_fused, v7d_swiglu_q8,
v7d_swiglu) without a GPU: exact integer group dots, the float accumulation
against float64, the reference's own swiglu validator against the oracle
behind the reference ABI, and the two documented corner cases (-128 weights,
the single-row path of v7d_swiglu)."""
from __future__ import annotations

import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
F = np.float32


def q8_case(rng, batch, n, d, wlim=127):
    xq = rng.integers(-127, 128, (batch, n), dtype=np.int8)
    xs = rng.uniform(0.001, 0.02, (batch, n // 64)).astype(F)
    wq = rng.integers(-wlim, wlim + 1, (d, n), dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, (d, n // 64)).astype(F)
    return xq, xs, wq, ws


def exact_q8(xq, xs, wq, ws):
    """float64 of sum_g (int dot_g) * ws_g * xs_g."""
    b, n = xq.shape
    d = wq.shape[0]
    dots = np.einsum("bgk,dgk->bdg", xq.reshape(b, n // 64, 64).astype(np.int64),
                     wq.reshape(d, n // 64, 64).astype(np.int64))
    return np.einsum("bdg,dg,bg->bd", dots.astype(np.float64), ws.astype(np.float64), xs.astype(np.float64))


@pytest.mark.parametrize("batch,n,d", [(1, 64, 1), (1, 1024, 37), (3, 2048, 256)])
def test_q8_gemv_vs_float64(oracle, batch, n, d):
    rng = np.random.default_rng(n + d)
    xq, xs, wq, ws = q8_case(rng, batch, n, d)
    got = oracle.q8_gemv(xq, xs, wq, ws)
    want = exact_q8(xq, xs, wq, ws)
    # fp32 accumulation over n/64 groups in 8 lane chains: error bound from the
    # magnitudes of the terms
    b, nn = xq.shape
    mag = np.einsum("bgk,dgk->bdg", np.abs(xq.reshape(b, nn // 64, 64).astype(np.int64)),
                    np.abs(wq.reshape(d, nn // 64, 64).astype(np.int64)))
    bound = np.einsum("bdg,dg,bg->bd", mag.astype(np.float64), ws.astype(np.float64), xs.astype(np.float64))
    assert np.all(np.abs(got - want) <= 1e-6 * bound * (nn // 64 + 8) + 1e-30)


def test_q8_gemv_integer_exact_when_scales_are_one(oracle):
    """With unit scales and few groups every partial sum is an exactly
    representable integer: the oracle must equal the integer dot."""
    rng = np.random.default_rng(5)
    xq, _, wq, _ = q8_case(rng, 2, 256, 9)
    xs = np.ones((2, 4), F)
    ws = np.ones((9, 4), F)
    got = oracle.q8_gemv(xq, xs, wq, ws)
    want = xq.astype(np.int64) @ wq.astype(np.int64).T
    assert np.array_equal(got, want.astype(F))


def test_neg128_weights_follow_vpsignb(oracle):
    """A -128 weight against a negative activation: vpsignb leaves -128, so
    the reference's product is |a| * (-128) -- 256 * a away from a * w."""
    n, d = 64, 2
    xq = np.zeros((1, n), np.int8)
    wq = np.zeros((d, n), np.int8)
    xq[0, :4] = [-3, 5, -128, 0]
    wq[0, :4] = [-128, -128, -128, -128]
    wq[1, :4] = [-127, -127, 127, 7]
    ones_x, ones_w = np.ones((1, 1), F), np.ones((d, 1), F)
    got = oracle.q8_gemv(xq, ones_x, wq, ones_w)
    true = xq.astype(np.int64) @ wq.astype(np.int64).T
    assert got[0, 0] == true[0, 0] + 256 * (-3) + 256 * (-128)
    assert got[0, 1] == true[0, 1]


def test_q8_fused_equals_quantize_then_gemv(oracle):
    rng = np.random.default_rng(9)
    x = rng.normal(0, 2, (2, 512)).astype(F)
    _, _, wq, ws = q8_case(rng, 1, 512, 40)
    q, s = oracle.quantize(x)
    assert np.array_equal(oracle.q8_fused_gemv(x, wq, ws), oracle.q8_gemv(q, s, wq, ws))


def test_swiglu_q8_gemv_is_swiglu_of_two_gemvs(oracle):
    rng = np.random.default_rng(11)
    xq, xs, gq, gs = q8_case(rng, 2, 1024, 50)
    _, _, uq, us = q8_case(rng, 2, 1024, 50)
    g = oracle.q8_gemv(xq, xs, gq, gs)
    u = oracle.q8_gemv(xq, xs, uq, us)
    with np.errstate(all="ignore"):
        assert np.array_equal(oracle.swiglu_q8_gemv(xq, xs, gq, gs, uq, us), oracle.swiglu(g, u))


@pytest.mark.parametrize("n", [64, 192, 256, 320, 448, 576, 2048])
def test_swiglu_f32q8_paths_agree_to_rounding(oracle, n):
    """The dual-row and single-row arithmetic of v7d_swiglu group the fp32
    sums differently; both stay within fp32 rounding of float64."""
    rng = np.random.default_rng(n)
    d = 33
    x = (0.1 + rng.integers(0, 100, (1, n)) / 1000).astype(F)
    gq = rng.integers(-100, 101, (d, n), dtype=np.int8)
    uq = rng.integers(-100, 101, (d, n), dtype=np.int8)
    gs = (0.1 + rng.integers(0, 100, (d, n // 64)) / 1000).astype(F)
    us = (0.1 + rng.integers(0, 100, (d, n // 64)) / 1000).astype(F)
    dual = oracle.swiglu_f32q8_gemv(x, gq, gs, uq, us)
    single = oracle.swiglu_f32q8_gemv(x, gq, gs, uq, us, single_row_path=True)

    def dot64(w, s):
        wf = w.astype(np.float64) * np.repeat(s.astype(np.float64), 64, axis=1)
        return x.astype(np.float64) @ wf.T

    g64, u64 = dot64(gq, gs), dot64(uq, us)
    want = g64 / (1 + np.exp(-g64)) * u64
    for got in (dual, single):
        assert np.allclose(got, want, rtol=2e-5, atol=1e-3)


def test_reference_swiglu_validator_on_oracle(oracle, tmp_path):
    """tools/v_swiglu_validate.cpp against the oracle: every F32xQ8 case passes
    (0.02 / 1e-4 against the double C reference) and every Q8xQ8 miss is one
    of the validator's documented float-vs-double known limits."""
    from oracle.pyoracle import ABI_SHIM
    exe = ROOT / "oracle" / "_ref" / "v_swiglu_validate"
    if not exe.exists():
        pytest.skip(f"{exe} not built")
    db = tmp_path / "empty.db"
    db.write_bytes(b"\n")
    r = subprocess.run([str(exe), str(ABI_SHIM), "--db", str(db)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:]
    assert re.search(r"F32xQ8 10 passed", r.stdout) and "0 hard failures" in r.stdout, r.stdout[-3000:]
