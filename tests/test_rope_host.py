"""The RoPE family without a GPU: the oracle's rope-only kernel and x87 table
builder against float64 restatements, and the library's host frequency
builder (v7g_rope_freqs, no device involved) against the oracle bit for bit."""
from __future__ import annotations

import math

import numpy as np
import pytest

F = np.float32
LLAMA3 = {"factor": 32.0, "high_freq_factor": 4.0, "low_freq_factor": 1.0, "orig_max_pos": 8192}


def llama3_freqs_f64(half: int, base: float, sc: dict) -> np.ndarray:
    """The published llama3 rope scaling (frequency-dependent: high
    frequencies kept, low ones divided by `factor`, a smooth blend between),
    in float64 -- an independent restatement of fused_f32_kernel.inc:186-256."""
    factor, hi, lo, old = sc["factor"], sc["high_freq_factor"], sc["low_freq_factor"], sc["orig_max_pos"]
    low_wl, high_wl = old / lo, old / hi
    out = []
    for j in range(half):
        inv = float(F(base)) ** (-j / half)
        wl = 2 * math.pi / inv
        if wl < high_wl:
            out.append(inv)
        elif wl > low_wl:
            out.append(inv / factor)
        else:
            s = (old / wl - lo) / (hi - lo)
            out.append((1 - s) * inv / factor + s * inv)
    return np.array(out)


@pytest.mark.parametrize("half", [16, 32, 64, 128, 256])
@pytest.mark.parametrize("base", [1e4, 5e5, 1e6])
def test_oracle_freqs_plain(oracle, half, base):
    f = oracle.rope_freqs(half, base)
    ref = float(F(base)) ** (-np.arange(half) / half)
    assert np.max(np.abs(f - ref) / ref) < 4e-16
    assert f[0] == 1.0


@pytest.mark.parametrize("half", [32, 64])
def test_oracle_freqs_llama3(oracle, half):
    f = oracle.rope_freqs(half, 5e5, LLAMA3)
    ref = llama3_freqs_f64(half, 5e5, LLAMA3)
    assert np.max(np.abs(f - ref) / ref) < 1e-14
    plain = oracle.rope_freqs(half, 5e5)
    assert f[0] == plain[0]                        # high frequency: unchanged
    assert f[-1] == pytest.approx(plain[-1] / 32)  # low frequency: divided by factor


def test_oracle_tables_vs_float64(oracle):
    """x87 tables against float64 sin/cos of the float64 angle: equal except
    where the two angle roundings straddle an fp32 rounding boundary."""
    P, half = 4096, 64
    c, s = oracle.rope_tables(P, half, half, 1e6)
    f = oracle.rope_freqs(half, 1e6)
    ang = np.arange(P, dtype=np.float64)[:, None] * f[None, :]
    for got, want in ((c, np.cos(ang)), (s, np.sin(ang))):
        assert np.max(np.abs(got - want)) <= 6e-8
        assert np.mean(got != want.astype(F)) < 1e-4
    assert np.array_equal(c[0], np.ones(half, F)) and np.array_equal(s[0], np.zeros(half, F))


def test_oracle_tables_offset_and_stride(oracle):
    c1, s1 = oracle.rope_tables(300, 32, 40, 1e6)
    c2, s2 = oracle.rope_tables(100, 32, 40, 1e6, pos0=200)
    assert np.array_equal(c1[200:], c2) and np.array_equal(s1[200:], s2)
    assert not c1[:, 32:].any() and not s1[:, 32:].any()


@pytest.mark.parametrize("pos0", [0, 3])
def test_oracle_rope_only_vs_float64(oracle, pos0):
    rng = np.random.default_rng(pos0)
    T, H, D = 9, 4, 128
    x = rng.normal(0, 1, (T, H, D)).astype(F)
    c, s = oracle.rope_tables(pos0 + T, D // 2, D // 2, 1e6)
    got = oracle.rope_only(x, c, s, pos0)
    lo, hi = x[..., :D // 2].astype(np.float64), x[..., D // 2:].astype(np.float64)
    cc = c[pos0:pos0 + T, None, :].astype(np.float64)
    ss = s[pos0:pos0 + T, None, :].astype(np.float64)
    want = np.concatenate([lo * cc - hi * ss, lo * ss + hi * cc], axis=-1)
    assert np.allclose(got, want, rtol=1e-6, atol=1e-6)
    if pos0 == 0:
        assert np.array_equal(got[0], x[0])


def test_oracle_rope_only_contract(oracle):
    x = np.zeros((1, 1, 48), F)
    c = np.zeros((2, 24), F)
    with pytest.raises(ValueError):
        oracle.rope_only(x, c, c, 1)


def test_library_host_freqs_equal_oracle(native_lib_path, oracle):
    """v7g_rope_freqs runs on the host (x87) and needs no device."""
    import v7multiplikator_b200 as v7g
    for sc in (None, LLAMA3):
        for half in (16, 32, 64, 128, 256):
            for base in (1e4, 5e5, 1e6):
                a, b = v7g.rope_freqs(half, base, sc), oracle.rope_freqs(half, base, sc)
                assert np.array_equal(a.view(np.int64), b.view(np.int64)), (sc, half, base)


def test_library_rope_argument_checks(native_lib_path):
    import v7multiplikator_b200 as v7g
    with pytest.raises(v7g.V7GError, match="half"):
        v7g.rope_freqs(300, 1e6)
    L = v7g.lib()
    assert L.v7g_rope_only_rows(1, 1, 4, 2, 2, 100, 1, 1, 0, 64, None) == v7g.ops.V7G_ERR_ARG
    assert L.v7g_rope_only_rows(1, 0, 4, 2, 0, 64, 0, 0, 0, 64, None) == v7g.ops.V7G_ERR_ARG  # NULL tables
    assert L.v7g_rope_only_rows(1, 0, 1, 2, 0, 64, 0, 0, 0, 64, None) == 0  # one token at position 0: nothing to do
    assert L.v7g_rope_tables(1, 1, 0, 10, 0, 0, 1, None) == v7g.ops.V7G_ERR_ARG
