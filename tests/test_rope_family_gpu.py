"""The rest of the RoPE family on the GPU, through the C-ABI: RoPE without the
norm (v7s_rope_only_heads, rope_only_kernel.inc:11-53), bit for bit against
the oracle, and the table builder (fused_f32_kernel.inc:117-302) against the
oracle's x87 tables (frequencies bit for bit; entries within one fp32 ulp,
all but a handful equal)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from test_parity_gpu import assert_same_f32, dev, host, normal

pytestmark = pytest.mark.gpu
F = np.float32

LLAMA3 = {"factor": 32.0, "high_freq_factor": 4.0, "low_freq_factor": 1.0, "orig_max_pos": 8192}


def ulp_distance(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    def key(x):
        i = np.asarray(x, F).view(np.int32).astype(np.int64)
        return np.where(i < 0, -(1 << 31) - i, i)
    return np.abs(key(a) - key(b))



def rope_tables_for(oracle, rng, rows, half, rmd, base):
    """cos/sin tables [rows, rmd]: the reference's own builder (x87, through the
    oracle) up to the 256 frequency pairs it makes; beyond that -- head_dim up to
    1024, which the kernels take with caller tables -- seeded unit-circle values."""
    if half <= 256:
        return oracle.rope_tables(rows, half, rmd, base)
    th = rng.uniform(-np.pi, np.pi, (rows, rmd))
    return np.cos(th).astype(np.float32), np.sin(th).astype(np.float32)

@pytest.mark.parametrize("head_dim", [32, 64, 96, 128, 256, 512, 1024])
@pytest.mark.parametrize("heads", [(16, 8), (5, 3), (0, 2), (4, 0)])
@pytest.mark.parametrize("tokens,pos0", [(1, 0), (1, 9), (7, 0), (130, 5)])
def test_rope_only_rows(cuda, oracle, head_dim, heads, tokens, pos0):
    import v7multiplikator_b200 as v7g
    hq, hk = heads
    rng = np.random.default_rng(head_dim * 1000 + hq * 10 + hk + tokens + pos0)
    q = normal(rng, (tokens, hq, head_dim))
    k = normal(rng, (tokens, hk, head_dim))
    cos, sin = rope_tables_for(oracle, rng, pos0 + tokens, head_dim // 2, head_dim, 1e6)
    qt, kt = dev(q), dev(k)
    v7g.rope_only_rows(qt if hq else None, kt if hk else None, dev(cos), dev(sin), pos0)
    if hq:
        assert_same_f32(host(qt), oracle.rope_only(q, cos, sin, pos0), "q")
    if hk:
        assert_same_f32(host(kt), oracle.rope_only(k, cos, sin, pos0), "k")
    if pos0 == 0 and hq:
        assert_same_f32(host(qt)[0], q[0], "position 0 is the identity")


def test_rope_only_unaligned_and_specials(cuda, oracle):
    """Misaligned tensors and table rows (the scalar kernel), and planted
    NaN / inf / subnormal values (FTZ+DAZ as the reference's workers)."""
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(7)
    tokens, hq, hk, d, rmd = 33, 3, 2, 64, 37  # rows of 37 floats: not 16-byte aligned
    q = normal(rng, (tokens, hq, d))
    k = normal(rng, (tokens, hk, d))
    q[3, 1, :6] = [np.nan, np.inf, -np.inf, 1e-39, -1e-39, 0.0]
    k[5, 0, 32:38] = [np.nan, np.inf, -np.inf, 1e-39, -1e-39, -0.0]
    cos, sin = oracle.rope_tables(tokens + 2, d // 2, rmd, 1e4)
    cos[4, 3] = 1e-39
    sin[6, 2] = -1e-39
    qbuf = torch.zeros(q.size + 1, device=cuda)
    kbuf = torch.zeros(k.size + 1, device=cuda)
    qt = qbuf[1:].view(tokens, hq, d)
    kt = kbuf[1:].view(tokens, hk, d)
    qt.copy_(dev(q))
    kt.copy_(dev(k))
    v7g.rope_only_rows(qt, kt, dev(cos), dev(sin), 2)
    with np.errstate(all="ignore"):
        assert_same_f32(host(qt), oracle.rope_only(q, cos, sin, 2), "q")
        assert_same_f32(host(kt), oracle.rope_only(k, cos, sin, 2), "k")


def test_v7s_rope_only_heads_per_token(cuda, oracle):
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(3)
    h, d, rmd = 8, 128, 64
    cos, sin = oracle.rope_tables(40, d // 2, rmd, 1e6)
    for pos in (0, 1, 39):
        buf = normal(rng, h * d)
        bt = dev(buf)
        v7g.v7s_rope_only_heads(bt, h, d, dev(cos), dev(sin), pos, rmd)
        assert_same_f32(host(bt), oracle.rope_only(buf.reshape(1, h, d), cos, sin, pos, rmd).reshape(-1))


def test_rope_only_full_size_c3_properties(cuda, oracle):
    """C3 geometry (Q [8192, 16, 128], K [8192, 8, 128]): sampled tokens bit
    for bit, and every pair's norm preserved to fp32 rounding."""
    import v7multiplikator_b200 as v7g
    T, D = 8192, 128
    q = torch.empty(T, 16, D, device=cuda)
    k = torch.empty(T, 8, D, device=cuda)
    v7g.fill_normal(q.view(T, -1), 21, 0.0, 1.0)
    v7g.fill_normal(k.view(T, -1), 22, 0.0, 1.0)
    q0, k0 = q.clone(), k.clone()
    cos, sin = v7g.rope_tables(T, D // 2, 1e6)
    v7g.rope_only_rows(q, k, cos, sin, 0)
    torch.cuda.synchronize()
    cos_h, sin_h = host(cos), host(sin)
    for t in (0, 1, 4095, 8191):
        want = oracle.rope_only(host(q0[t:t + 1]), cos_h, sin_h, t)
        assert_same_f32(host(q[t:t + 1]), want, f"token {t}")
    for before, after in ((q0, q), (k0, k)):
        b = before.double()
        a = after.double()
        nb = b[..., :D // 2] ** 2 + b[..., D // 2:] ** 2
        na = a[..., :D // 2] ** 2 + a[..., D // 2:] ** 2
        assert torch.allclose(na, nb, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("base,scaling", [(1e6, None), (1e4, None), (5e5, LLAMA3)])
def test_rope_tables_match_x87(cuda, oracle, base, scaling):
    """The device table kernel against the oracle's x87 fsincos tables at the
    reference's full size (131072 positions, half 64)."""
    import v7multiplikator_b200 as v7g
    P, half = 131072, 64
    cos, sin = v7g.rope_tables(P, half, base, scaling=scaling)
    want_c, want_s = oracle.rope_tables(P, half, half, base, scaling=scaling)
    got_c, got_s = host(cos), host(sin)
    for got, want, what in ((got_c, want_c, "cos"), (got_s, want_s, "sin")):
        d = ulp_distance(got, want)
        assert d.max() <= 1, f"{what}: max ulp distance {d.max()}"
        assert (d > 0).sum() <= 16, f"{what}: {(d > 0).sum()} entries off by one ulp"
    assert np.array_equal(got_c[0], np.ones(half, F)) and np.array_equal(got_s[0], np.zeros(half, F))


def test_rope_tables_offset_stride_and_zero_columns(cuda, oracle):
    import v7multiplikator_b200 as v7g
    cos, sin = v7g.rope_tables(100, 48, 1e6, stride=52, pos0=1000)
    want_c, want_s = oracle.rope_tables(100, 48, 52, 1e6, pos0=1000)
    assert (ulp_distance(host(cos), want_c) <= 1).all() and (ulp_distance(host(sin), want_s) <= 1).all()
    assert not host(cos)[:, 48:].any() and not host(sin)[:, 48:].any()


def test_rope_init_builds_library_tables(cuda):
    import v7multiplikator_b200 as v7g
    cos, sin = v7g.rope_init(128, 1e6)
    assert cos.shape == (131072, 64) and sin.shape == (131072, 64)
    want_c, want_s = v7g.rope_tables(131072, 64, 1e6)
    torch.cuda.synchronize()
    assert torch.equal(cos, want_c) and torch.equal(sin, want_s)
    cos2, _ = v7g.rope_init(64, 5e5, LLAMA3)
    assert cos2.shape == (131072, 32)
    want_c2, _ = v7g.rope_tables(131072, 32, 5e5, scaling=LLAMA3)
    torch.cuda.synchronize()
    assert torch.equal(cos2, want_c2)


def test_rope_only_rejects_bad_head_dim(cuda):
    import v7multiplikator_b200 as v7g
    q = torch.zeros(2, 2, 48, device=cuda)
    t = torch.zeros(4, 24, device=cuda)
    with pytest.raises(v7g.V7GError, match="multiple of 32"):
        v7g.rope_only_rows(q, None, t, t, 1)


def test_rope_entries_reject_head_dim_above_1024(cuda):
    """One 32-block past the largest head the kernels take (1024) is refused
    by both entries, with the range named, before anything is launched."""
    import v7multiplikator_b200 as v7g
    q = torch.zeros(2, 1, 1056, device=cuda)
    t = torch.zeros(4, 528, device=cuda)
    w = torch.ones(1056, device=cuda)
    with pytest.raises(v7g.V7GError, match=r"\[32, 1024\]"):
        v7g.rope_only_rows(q, None, t, t, 1)
    with pytest.raises(v7g.V7GError, match=r"\[32, 1024\]"):
        v7g.rmsnorm_rope_rows(q, None, w, None, t, t, 1, 1e-6)


def test_reference_abi_rope_entries(cuda, oracle, tmp_path):
    """v7s_rope_only_heads, v7s_qk_fork_heads and v7s_rope_init through the
    Microsoft x64 convention from C (tests/abi_probe.c, gpu mode); the probe's
    RMSNorm+RoPE over the library's own device tables is then checked against
    the oracle with the oracle's x87 tables."""
    import subprocess
    from pathlib import Path
    import os
    root = Path(__file__).resolve().parent.parent
    exe = tmp_path / "abi_probe"
    subprocess.run(["gcc", "-O1", "-std=c11", f"-I{root / 'include'}", str(root / "tests" / "abi_probe.c"), "-o",
                    str(exe), "-ldl", "-lm"], check=True)
    import v7multiplikator_b200 as v7g
    out = tmp_path / "probe.bin"
    r = subprocess.run([str(exe), str(v7g.LIB_PATH), str(root / "tests" / "golden" / "v7_load_names.txt"), "gpu"],
                       capture_output=True, text=True, timeout=300, env={**os.environ, "V7G_PROBE_OUT": str(out)})
    assert r.returncode == 0 and "PROBE PASSED" in r.stdout, r.stdout + r.stderr
    raw = np.fromfile(out, F)
    H, D, pos = 4, 64, 5
    buf, w, got = raw[:H * D], raw[H * D:H * D + D], raw[H * D + D:]
    cos, sin = oracle.rope_tables(pos + 1, D // 2, D // 2, 1e6)
    assert_same_f32(got, oracle.rope(buf.reshape(1, H, D), w, cos, sin, pos, 1e-6).reshape(-1))
