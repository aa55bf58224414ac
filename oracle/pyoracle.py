"""numpy front end of the C oracle (oracle/v7_oracle.c) -- TEST INFRASTRUCTURE ONLY.

Used as the parity checker by tests/, __graft_entry__.smoke() and the CPU
baseline of bench.py.  ``ensure_built()`` compiles the library with the recipe
in oracle/Makefile when it is missing.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, c_double, c_float, c_int, c_int64, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libv7_oracle.so"
ABI_SHIM = HERE / "_build" / "libv7_oracle_abi.so"
REF_DIR = HERE / "_ref"


def ensure_built() -> None:
    if not LIB.exists() or not ABI_SHIM.exists():
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def _ptr(a: np.ndarray) -> c_void_p:
    assert a.flags["C_CONTIGUOUS"]
    return c_void_p(a.ctypes.data)


class Oracle:
    """Thin typed wrapper; every method allocates and returns its outputs."""

    def __init__(self, nthreads: int | None = None):
        ensure_built()
        self.lib = ctypes.CDLL(str(LIB))
        self.nthreads = nthreads or max(1, os.cpu_count() or 1)
        L = self.lib
        sig = {
            "orc_rmsnorm_rows": [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_float, c_int],
            "orc_fused_add_rmsnorm_rows": [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_float, c_int],
            "orc_rmsnorm_rope_rows": [c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int64, c_int,
                                      c_float, c_int],
            "orc_swiglu": [c_void_p, c_void_p, c_void_p, c_int64, c_int],
            "orc_quantize_rows": [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int],
            "orc_swiglu_q8_rows": [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int],
            "orc_add_inplace": [c_void_p, c_void_p, c_int64, c_int],
            "orc_rmsnorm_quantize_rows": [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_float, c_int],
            "orc_rope_only_rows": [c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p, c_int64, c_int, c_int],
            "orc_rope_freqs": [c_void_p, c_int, c_float, c_int, c_float, c_float, c_float, c_int],
            "orc_fill_normal": [c_void_p, c_int64, c_int64, c_int64, ctypes.c_uint64, c_float, c_float, c_int],
            "orc_swiglu_q8_rows_avx2": [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int],
            "orc_rope_tables": [c_void_p, c_void_p, c_int64, c_int64, c_int, c_int, c_void_p, c_int],
            "orc_q8_gemv": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_int],
            "orc_q8_fused_gemv": [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_int],
            "orc_swiglu_q8_gemv": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int,
                                   c_int, c_int],
            "orc_swiglu_f32q8_gemv": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int,
                                      c_int, c_int],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = c_int
        L.orc_sigmoid.argtypes = [c_float]
        L.orc_sigmoid.restype = c_float

    @staticmethod
    def _ok(rc: int, what: str) -> None:
        if rc != 0:
            raise ValueError(f"oracle {what}: contract violation")

    def rmsnorm(self, x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        rows, n = x.reshape(-1, x.shape[-1]).shape
        o = np.empty_like(x)
        self._ok(self.lib.orc_rmsnorm_rows(_ptr(o), _ptr(x), _ptr(np.ascontiguousarray(w, np.float32)), rows, n, eps,
                                           self.nthreads), "rmsnorm")
        return o

    def fused_add_rmsnorm(self, r: np.ndarray, a: np.ndarray, w: np.ndarray, eps: float):
        """Returns (out, residual after the in-place add)."""
        r = np.array(r, np.float32, copy=True, order="C")
        a = np.ascontiguousarray(a, np.float32)
        rows, n = r.reshape(-1, r.shape[-1]).shape
        o = np.empty_like(r)
        self._ok(self.lib.orc_fused_add_rmsnorm_rows(_ptr(o), _ptr(r), _ptr(a), _ptr(np.ascontiguousarray(w, np.float32)),
                                                     rows, n, eps, self.nthreads), "fused_add_rmsnorm")
        return o, r

    def rope(self, buf: np.ndarray, w: np.ndarray, cos: np.ndarray, sin: np.ndarray, pos0: int, eps: float,
             rope_max_dim: int | None = None) -> np.ndarray:
        """buf [tokens, heads, head_dim]; cos/sin flat tables with rows of
        rope_max_dim (default: the last dimension of cos)."""
        out = np.array(buf, np.float32, copy=True, order="C")
        tokens, heads, hd = out.shape
        cos = np.ascontiguousarray(cos, np.float32)
        sin = np.ascontiguousarray(sin, np.float32)
        rmd = rope_max_dim if rope_max_dim is not None else cos.shape[-1]
        self._ok(self.lib.orc_rmsnorm_rope_rows(_ptr(out), tokens, heads, hd, _ptr(np.ascontiguousarray(w, np.float32)),
                                                _ptr(cos), _ptr(sin), pos0, rmd, eps, self.nthreads), "rope")
        return out

    def sigmoid(self, g: float) -> float:
        return float(self.lib.orc_sigmoid(g))

    def swiglu(self, g: np.ndarray, u: np.ndarray) -> np.ndarray:
        g = np.ascontiguousarray(g, np.float32)
        u = np.ascontiguousarray(u, np.float32)
        o = np.empty_like(g)
        self._ok(self.lib.orc_swiglu(_ptr(o), _ptr(g), _ptr(u), g.size, self.nthreads), "swiglu")
        return o

    def quantize(self, x: np.ndarray):
        """Per-row Q8 of x [rows, n] -> (codes int8 [rows, n], scales [rows, ceil(n/64)])."""
        x = np.ascontiguousarray(x, np.float32)
        x2 = x.reshape(-1, x.shape[-1])
        rows, n = x2.shape
        q = np.empty((rows, n), np.int8)
        s = np.empty((rows, (n + 63) // 64), np.float32)
        self._ok(self.lib.orc_quantize_rows(_ptr(q), _ptr(s), _ptr(x2), rows, n, self.nthreads), "quantize")
        return q, s

    def swiglu_q8(self, g: np.ndarray, u: np.ndarray, out: tuple[np.ndarray, np.ndarray] | None = None):
        """SwiGLU then Q8 per row -> (codes int8 [rows, n], scales [rows, n/64]);
        `out` = preallocated (codes, scales) to write instead."""
        g = np.ascontiguousarray(g, np.float32)
        u = np.ascontiguousarray(u, np.float32)
        rows, n = g.reshape(-1, g.shape[-1]).shape
        if out is None:
            q = np.empty((rows, n), np.int8)
            s = np.empty((rows, n // 64), np.float32)
        else:
            q, s = out
            assert q.shape == (rows, n) and q.dtype == np.int8 and s.shape == (rows, n // 64) and s.dtype == np.float32
        self._ok(self.lib.orc_swiglu_q8_rows(_ptr(q), _ptr(s), _ptr(g), _ptr(u), rows, n, self.nthreads), "swiglu_q8")
        return q, s

    def swiglu_q8_avx2(self, g: np.ndarray, u: np.ndarray, out: tuple[np.ndarray, np.ndarray] | None = None):
        """swiglu_q8 in AVX2 (the reference's instruction forms, eight lanes
        at a time): identical bits, the form the CPU baseline times."""
        g = np.ascontiguousarray(g, np.float32)
        u = np.ascontiguousarray(u, np.float32)
        rows, n = g.reshape(-1, g.shape[-1]).shape
        if out is None:
            q = np.empty((rows, n), np.int8)
            s = np.empty((rows, n // 64), np.float32)
        else:
            q, s = out
            assert q.shape == (rows, n) and q.dtype == np.int8 and s.shape == (rows, n // 64) and s.dtype == np.float32
        self._ok(self.lib.orc_swiglu_q8_rows_avx2(_ptr(q), _ptr(s), _ptr(g), _ptr(u), rows, n, self.nthreads), "swiglu_q8_avx2")
        return q, s

    def fill_normal(self, rows: int, n: int, row0: int = 0, seed: int = 0, mean: float = 0.0, std: float = 1.0,
                    out: np.ndarray | None = None) -> np.ndarray:
        """The library's synthetic generator (v7g_fill_normal) on the CPU: rows
        row0 .. row0 + rows - 1 of the N(mean, std) matrix keyed by `seed`,
        bit-identical to the device's."""
        o = np.empty((rows, n), np.float32) if out is None else out
        assert o.shape == (rows, n) and o.dtype == np.float32 and o.flags["C_CONTIGUOUS"]
        self._ok(self.lib.orc_fill_normal(_ptr(o), rows, n, row0, seed, mean, std, self.nthreads), "fill_normal")
        return o

    def add_inplace(self, x: np.ndarray, y: np.ndarray) -> np.ndarray:
        out = np.array(x, np.float32, copy=True, order="C")
        self._ok(self.lib.orc_add_inplace(_ptr(out), _ptr(np.ascontiguousarray(y, np.float32)), out.size,
                                          self.nthreads), "add_inplace")
        return out

    def rmsnorm_quantize(self, x: np.ndarray, w: np.ndarray, eps: float):
        x = np.ascontiguousarray(x, np.float32)
        rows, n = x.reshape(-1, x.shape[-1]).shape
        q = np.empty((rows, n), np.int8)
        s = np.empty((rows, n // 64), np.float32)
        self._ok(self.lib.orc_rmsnorm_quantize_rows(_ptr(q), _ptr(s), _ptr(x), _ptr(np.ascontiguousarray(w, np.float32)),
                                                    rows, n, eps, self.nthreads), "rmsnorm_quantize")
        return q, s

    def rope_only(self, buf: np.ndarray, cos: np.ndarray, sin: np.ndarray, pos0: int,
                  rope_max_dim: int | None = None) -> np.ndarray:
        """RoPE without the norm; buf [tokens, heads, head_dim]."""
        out = np.array(buf, np.float32, copy=True, order="C")
        tokens, heads, hd = out.shape
        cos = np.ascontiguousarray(cos, np.float32)
        sin = np.ascontiguousarray(sin, np.float32)
        rmd = rope_max_dim if rope_max_dim is not None else cos.shape[-1]
        self._ok(self.lib.orc_rope_only_rows(_ptr(out), tokens, heads, hd, _ptr(cos), _ptr(sin), pos0, rmd,
                                             self.nthreads), "rope_only")
        return out

    def rope_freqs(self, half: int, base: float = 1e6, scaling: dict | None = None) -> np.ndarray:
        """freqs[j] (float64) as the reference's table builder stores them;
        scaling = None or {"factor", "high_freq_factor", "low_freq_factor",
        "orig_max_pos"} for llama3 scaling."""
        f = np.empty(half, np.float64)
        sc = scaling or {}
        self._ok(self.lib.orc_rope_freqs(_ptr(f), half, base, 1 if scaling else 0, sc.get("factor", 0.0),
                                         sc.get("high_freq_factor", 0.0), sc.get("low_freq_factor", 0.0),
                                         int(sc.get("orig_max_pos", 0))), "rope_freqs")
        return f

    def rope_tables(self, positions: int, half: int, stride: int | None = None, base: float = 1e6,
                    pos0: int = 0, scaling: dict | None = None):
        """cos, sin [positions, stride] fp32 for positions pos0.. (x87, as the
        reference builds them)."""
        stride = stride or half
        freqs = self.rope_freqs(half, base, scaling)
        c = np.empty((positions, stride), np.float32)
        s = np.empty((positions, stride), np.float32)
        self._ok(self.lib.orc_rope_tables(_ptr(c), _ptr(s), pos0, positions, half, stride, _ptr(freqs),
                                          self.nthreads), "rope_tables")
        return c, s

    # ---- Q8-weight GEMVs: activations [batch, n], weights [d, n] + [d, n/64]

    @staticmethod
    def _c(a, dt):
        return np.ascontiguousarray(a, dt)

    def q8_gemv(self, xq, xs, wq, ws) -> np.ndarray:
        xq, xs, wq, ws = self._c(xq, np.int8), self._c(xs, np.float32), self._c(wq, np.int8), self._c(ws, np.float32)
        batch, n = xq.reshape(-1, xq.shape[-1]).shape
        d = wq.shape[0]
        out = np.empty((batch, d), np.float32)
        self._ok(self.lib.orc_q8_gemv(_ptr(out), _ptr(xq), _ptr(xs), _ptr(wq), _ptr(ws), batch, n, d, self.nthreads),
                 "q8_gemv")
        return out

    def q8_fused_gemv(self, x, wq, ws) -> np.ndarray:
        x, wq, ws = self._c(x, np.float32), self._c(wq, np.int8), self._c(ws, np.float32)
        batch, n = x.reshape(-1, x.shape[-1]).shape
        d = wq.shape[0]
        out = np.empty((batch, d), np.float32)
        self._ok(self.lib.orc_q8_fused_gemv(_ptr(out), _ptr(x), _ptr(wq), _ptr(ws), batch, n, d, self.nthreads),
                 "q8_fused_gemv")
        return out

    def swiglu_q8_gemv(self, xq, xs, gq, gs, uq, us) -> np.ndarray:
        xq, xs = self._c(xq, np.int8), self._c(xs, np.float32)
        gq, gs, uq, us = self._c(gq, np.int8), self._c(gs, np.float32), self._c(uq, np.int8), self._c(us, np.float32)
        batch, n = xq.reshape(-1, xq.shape[-1]).shape
        d = gq.shape[0]
        out = np.empty((batch, d), np.float32)
        self._ok(self.lib.orc_swiglu_q8_gemv(_ptr(out), _ptr(xq), _ptr(xs), _ptr(gq), _ptr(gs), _ptr(uq), _ptr(us),
                                             batch, n, d, self.nthreads), "swiglu_q8_gemv")
        return out

    def swiglu_f32q8_gemv(self, x, gq, gs, uq, us, single_row_path: bool = False) -> np.ndarray:
        x = self._c(x, np.float32)
        gq, gs, uq, us = self._c(gq, np.int8), self._c(gs, np.float32), self._c(uq, np.int8), self._c(us, np.float32)
        batch, n = x.reshape(-1, x.shape[-1]).shape
        d = gq.shape[0]
        out = np.empty((batch, d), np.float32)
        self._ok(self.lib.orc_swiglu_f32q8_gemv(_ptr(out), _ptr(x), _ptr(gq), _ptr(gs), _ptr(uq), _ptr(us), batch, n, d,
                                                int(single_row_path), self.nthreads), "swiglu_f32q8_gemv")
        return out
