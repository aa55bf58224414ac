"""The oracle against the reference's own C reference kernels
(tests/golden/kt_cref.npz, written by tests/golden/make_golden.py from
tools/kt_utils.h) on every case the reference's validators run, with the
validators' tolerances:

  rmsnorm / rmsnorm_rope / add+rmsnorm  1e-3 abs  (kt_utils.h:820, :976, :1063)
  add_inplace                           1e-6 abs  (kt_utils.h:1010)
  quantize codes                        bit-exact (kt_utils.h:703-730)

The reference validators read eps from the library; the C references here ran
with eps = 1e-6 (rope cases: their own eps column).
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

import reffills as rf

RMS_SIZES = [64, 128, 256, 1024, 2048, 3072, 8192]
ADD_RMS_SIZES = [8, 16, 24, 48, 64, 128, 256, 1024, 2048, 3072, 8192]
ROPE_CASES = [(1, 64, 0, 64, 1e-6), (1, 64, 7, 64, 1e-6), (4, 64, 0, 64, 1e-6), (4, 64, 31, 64, 1e-6),
              (8, 64, 7, 64, 1e-6), (8, 128, 0, 128, 1e-6), (16, 64, 0, 64, 1e-6), (16, 64, 31, 64, 1e-6),
              (32, 64, 7, 64, 1e-6), (32, 128, 0, 128, 1e-6), (40, 64, 31, 64, 1e-6), (40, 128, 7, 128, 1e-6),
              (32, 64, 0, 64, 1e-5), (32, 64, 31, 64, 1e-5), (8, 64, 7, 64, 1e-5)]
ADD_SIZES = [32, 64, 96, 128, 160, 1024, 2048]
Q_SIZES = [64, 256, 1024, 4096, 8192, 65536]
SEEDS = [12345, 67890]
Q_SEEDS = [12345, 67890, 11111]
EPS = 1e-6


def rope_key(h, d, pos, rmd, eps, seed):
    return f"{h}x{d}/{pos}/{rmd}/{'1e-5' if eps == 1e-5 else '1e-6'}/{seed}"


@pytest.mark.parametrize("seed", SEEDS)
@pytest.mark.parametrize("size", RMS_SIZES)
def test_rmsnorm_vs_cref(oracle, golden, size, seed):
    x, w = rf.rmsnorm_case(size, seed)
    out = oracle.rmsnorm(x[None], w, EPS)[0]
    ref = golden[f"rmsnorm/{size}/{seed}"]
    assert np.max(np.abs(out - ref)) <= 1e-3


@pytest.mark.parametrize("seed", SEEDS)
@pytest.mark.parametrize("dim", ADD_RMS_SIZES)
def test_fused_add_rmsnorm_vs_cref(oracle, golden, dim, seed):
    r, a, w = rf.add_rmsnorm_case(dim, seed)
    out, res = oracle.fused_add_rmsnorm(r[None], a[None], w, EPS)
    assert np.max(np.abs(out[0] - golden[f"add_rmsnorm/{dim}/{seed}"])) <= 1e-3
    # the residual add is a single rounding in both: bit-exact
    assert np.array_equal(res[0], golden[f"add_rmsnorm_res/{dim}/{seed}"])


@pytest.mark.parametrize("seed", SEEDS)
@pytest.mark.parametrize("case", ROPE_CASES, ids=lambda c: f"{c[0]}x{c[1]}-pos{c[2]}-eps{c[4]}")
def test_rmsnorm_rope_vs_cref(oracle, golden, case, seed):
    h, d, pos, rmd, eps = case
    key = rope_key(h, d, pos, rmd, eps, seed)
    buf, w = rf.rope_case(h, d, seed)
    cos = golden[f"rope_cos/{key}"]
    sin = golden[f"rope_sin/{key}"]
    # one token at position pos: the rows entry with pos0 = pos reads row pos
    out = oracle.rope(buf.reshape(1, h, d), w, cos, sin, pos, eps, rope_max_dim=rmd)
    assert np.max(np.abs(out.reshape(-1) - golden[f"rope/{key}"])) <= 1e-3


@pytest.mark.parametrize("seed", SEEDS)
@pytest.mark.parametrize("n", ADD_SIZES)
def test_add_inplace_vs_cref(oracle, golden, n, seed):
    x, y = rf.add_inplace_case(n, seed)
    out = oracle.add_inplace(x, y)
    ref = golden[f"add_inplace/{n}/{seed}"]
    assert np.max(np.abs(out - ref)) <= 1e-6
    assert np.array_equal(out, ref)


@pytest.mark.parametrize("seed", Q_SEEDS)
@pytest.mark.parametrize("n", Q_SIZES)
@pytest.mark.parametrize("pattern", range(7), ids=rf.QUANT_PATTERNS)
def test_quantize_vs_cref(oracle, golden, pattern, n, seed):
    x = rf.quantize_pattern(n, seed, pattern)
    q, s = oracle.quantize(x[None])
    key = f"{pattern}/{n}/{seed}"
    digest = bytes(golden[f"quant_codes_sha256/{key}"]).decode()
    assert hashlib.sha256(q.tobytes()).hexdigest() == digest
    ref_s = golden[f"quant_scales/{key}"]
    if pattern == 2:
        # all-zero groups: the C reference uses 1/127, the reference's AVX2
        # kernel floors wmax at 127 * 2^-126, i.e. scale = FLT_MIN
        # (quantize_kernel.inc:40-41, :84); codes agree (all zero).
        assert np.all(s[0] == np.float32(np.finfo(np.float32).tiny))
    else:
        np.testing.assert_array_equal(s[0], ref_s)
