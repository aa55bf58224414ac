"""Input fills of the reference's validators, regenerated with glibc rand().

The reference's validators seed glibc's srand() and draw rand() in a fixed
order (tools/kt_utils.h).  Calling the same libc functions through ctypes and
doing the float arithmetic in float32 reproduces their inputs bit for bit, so
the golden outputs of tests/golden/kt_cref.npz apply to them.
"""
from __future__ import annotations

import ctypes

import numpy as np

_libc = ctypes.CDLL("libc.so.6")
_libc.rand.restype = ctypes.c_int
_libc.srand.argtypes = [ctypes.c_uint]

F = np.float32


def srand(seed: int) -> None:
    _libc.srand(seed)


def rand_ints(count: int) -> np.ndarray:
    return np.fromiter((_libc.rand() for _ in range(count)), dtype=np.int64, count=count)


def uniform_pm1(count: int) -> np.ndarray:
    """-1.0f + (float)(rand() % 2001) / 1000.0f (kt_utils.h:812-816)."""
    r = rand_ints(count) % 2001
    return (F(-1.0) + r.astype(F) / F(1000.0)).astype(F)


def uniform_weight(count: int) -> np.ndarray:
    """0.5f + (float)(rand() % 1001) / 1000.0f (kt_utils.h:815-816)."""
    r = rand_ints(count) % 1001
    return (F(0.5) + r.astype(F) / F(1000.0)).astype(F)


def uniform_pm10(count: int) -> np.ndarray:
    """-10.0f + (float)(rand() % 20001) / 1000.0f (kt_utils.h:1001-1005)."""
    r = rand_ints(count) % 20001
    return (F(-10.0) + r.astype(F) / F(1000.0)).astype(F)


def rmsnorm_case(size: int, seed: int):
    """x, weight of kt_verify_rmsnorm (kt_utils.h:797-830)."""
    srand(seed)
    x = uniform_pm1(size)
    w = uniform_weight(size)
    return x, w


def add_rmsnorm_case(dim: int, seed: int):
    """residual, add, weight of kt_verify_fused_add_rmsnorm (kt_utils.h:1049-1057)."""
    srand(seed)
    r = uniform_pm1(dim)
    a = uniform_pm1(dim)
    w = uniform_weight(dim)
    return r, a, w


def rope_case(n_heads: int, head_dim: int, seed: int):
    """buf, norm_weight of kt_verify_rmsnorm_rope_heads (kt_utils.h:953-957);
    the tables are stored in the golden fixture."""
    srand(seed)
    buf = uniform_pm1(n_heads * head_dim)
    w = uniform_weight(head_dim)
    return buf, w


def add_inplace_case(n: int, seed: int):
    """x, y of kt_verify_add_inplace (kt_utils.h:1001-1005)."""
    srand(seed)
    x = uniform_pm10(n)
    y = uniform_pm10(n)
    return x, y


QUANT_PATTERNS = ["small_pos", "wide_rand", "all_zero", "alternating", "ramp", "large_mix", "positional"]


def quantize_pattern(n: int, seed: int, pattern: int) -> np.ndarray:
    """kt_init_quantize_pattern (kt_utils.h:151-191)."""
    srand(seed)
    i = np.arange(n, dtype=np.int64)
    if pattern == 0:
        return (F(0.1) + (rand_ints(n) % 100).astype(F) / F(1000.0)).astype(F)
    if pattern == 1:
        return ((rand_ints(n) % 10000 - 5000).astype(F) / F(1000.0)).astype(F)
    if pattern == 2:
        return np.zeros(n, F)
    if pattern == 3:
        return np.where(i % 2 == 0, F(1.0), F(-1.0)).astype(F)
    if pattern == 4:
        return (i % 64).astype(F)
    if pattern == 5:
        return ((rand_ints(n) % 100000 - 50000).astype(F) / F(1000.0)).astype(F)
    if pattern == 6:
        return ((i % 64) - 32).astype(F)
    return np.ones(n, F)
