"""Python host layer over the native library's C-ABI (include/v7g.h).

Each function takes torch CUDA tensors, checks shapes/dtypes/devices on the
host and calls one ``v7g_*`` entry through ctypes on the tensor's current CUDA
stream.  Nothing here computes: the work is done by the sm_100a kernels in
``lib/libv7_threading.so``, and the import fails loudly when that library is
missing.  Errors raise :class:`V7GError` with the library's message.

Two families mirror the reference's operator interface:

* row-batched ops (``rmsnorm_rows`` & co.) -- the device-resident, batched form
  of v7's per-vector kernels, one launch for all rows;
* per-vector ops named after the reference exports (``v7s_rmsnorm``,
  ``v7s_add_inplace``, ``v7s_fused_add_rmsnorm``, ``v7s_rmsnorm_rope_heads``,
  ``v7s_rope_only_heads``, ``v7d_quantize``, ``v7s_rmsnorm_quantize``) with the reference's argument
  meaning (src/v7_lib.h:123-124, :270-273): one vector or one token per call,
  RMS epsilon taken from the library global (``set_rms_eps``), like the
  reference's BSS ``g_rms_eps``.
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int64, c_uint64, c_void_p, c_char_p
from pathlib import Path
from typing import Optional

import torch

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libv7_threading.so"

V7G_OK = 0
V7G_ERR_ARG = 1
V7G_ERR_CUDA = 2
V7G_ERR_UNSUPPORTED = 3
V7G_ERR_NO_DEVICE = 4


class V7GError(RuntimeError):
    """A v7g entry point returned a non-zero status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[v7g status {code}] {message}")
        self.code = code


_SIGNATURES = {
    "v7g_rmsnorm_rows": [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_float, c_void_p],
    "v7g_fused_add_rmsnorm_rows": [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_float, c_void_p],
    "v7g_rmsnorm_rope_rows": [c_void_p, c_void_p, c_int64, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p,
                              c_void_p, c_int64, c_int, c_float, c_void_p],
    "v7g_swiglu": [c_void_p, c_void_p, c_void_p, c_int64, c_void_p],
    "v7g_swiglu_q8_rows": [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p],
    "v7g_quantize_rows": [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p],
    "v7g_add_inplace": [c_void_p, c_void_p, c_int64, c_void_p],
    "v7g_rmsnorm_quantize_rows": [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_float, c_void_p],
    "v7g_fill_normal": [c_void_p, c_int64, c_int64, c_int64, c_uint64, c_float, c_float, c_void_p],
    "v7g_selftest_arith": [c_void_p, c_void_p],
    "v7g_rope_only_rows": [c_void_p, c_void_p, c_int64, c_int, c_int, c_int, c_void_p, c_void_p, c_int64, c_int,
                           c_void_p],
    "v7g_rope_freqs": [c_void_p, c_int, c_float, c_int, c_float, c_float, c_float, c_int],
    "v7g_rope_tables": [c_void_p, c_void_p, c_int64, c_int64, c_int, c_int, c_void_p, c_void_p],
    "v7g_rope_init": [c_int, c_float, c_int, c_float, c_float, c_float, c_int],
    "v7g_get_rope_tables": [c_void_p, c_void_p, c_void_p],
    "v7g_q8_gemv": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_void_p],
    "v7g_q8_fused_gemv": [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_void_p],
    "v7g_swiglu_q8_gemv": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int,
                           c_void_p],
    "v7g_swiglu_f32q8_gemv": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int,
                              c_void_p],
    "v7g_rmsnorm_rows_noalloc": [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_float, c_void_p],
}

# Size of the static device staging array of rmsnorm_rows_noalloc (per GPU).
NOALLOC_SCRATCH_BYTES = 4 << 20

# Positions of the tables rope_init builds (V7G_ROPE_TABLE_POSITIONS).
ROPE_TABLE_POSITIONS = 131072

_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    """The loaded native library (loaded once).  Raises if it was not built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"v7g native library {LIB_PATH} is missing; build it with "
                "`python -m v7multiplikator_b200.build` (needs nvcc)")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, args in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = c_int
        L.v7g_set_rms_eps.argtypes = [c_float]
        L.v7g_set_rms_eps.restype = None
        L.v7g_get_rms_eps.argtypes = []
        L.v7g_get_rms_eps.restype = c_float
        L.v7g_last_error.restype = c_char_p
        L.v7g_launch_count.restype = c_uint64
        L.v7g_set_launch_overlap.argtypes = [c_int]
        L.v7g_set_launch_overlap.restype = None
        L.v7g_get_launch_overlap.argtypes = []
        L.v7g_get_launch_overlap.restype = c_int
        L.v7g_version.restype = c_char_p
        L.v7g_pipeline_timeouts.restype = ctypes.c_uint
        _lib = L
    return _lib


def _check(rc: int) -> None:
    if rc != V7G_OK:
        raise V7GError(rc, lib().v7g_last_error().decode(errors="replace"))


def _stream(t: torch.Tensor, stream: Optional[torch.cuda.Stream]) -> int:
    s = stream if stream is not None else torch.cuda.current_stream(t.device)
    return s.cuda_stream


def _want(t: Optional[torch.Tensor], name: str, dtype: torch.dtype, device: torch.device) -> int:
    if t is None:
        return 0
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if t.device != device or t.device.type != "cuda":
        raise ValueError(f"{name} must be on {device}, got {t.device}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t.data_ptr()


def _rows(x: torch.Tensor) -> tuple[int, int]:
    if x.dim() < 1:
        raise ValueError("expected at least one dimension")
    n = x.shape[-1]
    return (x.numel() // n if n else 0), n


# ---------------------------------------------------------------- row-batched


def rmsnorm_rows(out: torch.Tensor, x: torch.Tensor, weight: torch.Tensor, eps: float,
                 stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """out[r] = (x[r] * s_r) * weight, s_r = 1/sqrt(mean(x[r]^2) + eps); rows = all
    leading dims of x (v7s_rmsnorm per row, rmsnorm_kernel.inc:12-75)."""
    rows, n = _rows(x)
    d = x.device
    if out.shape != x.shape or weight.numel() != n:
        raise ValueError("shape mismatch")
    _check(lib().v7g_rmsnorm_rows(_want(out, "out", torch.float32, d), _want(x, "x", torch.float32, d),
                                  _want(weight, "weight", torch.float32, d), rows, n, eps, _stream(x, stream)))
    return out


def fused_add_rmsnorm_rows(out: torch.Tensor, residual: torch.Tensor, add: torch.Tensor, weight: torch.Tensor,
                           eps: float, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """residual += add (in place); out = rmsnorm(residual) * weight, per row
    (v7s_fused_add_rmsnorm, add_rmsnorm_kernel.inc:15-129)."""
    rows, n = _rows(residual)
    d = residual.device
    if out.shape != residual.shape or add.shape != residual.shape or weight.numel() != n:
        raise ValueError("shape mismatch")
    _check(lib().v7g_fused_add_rmsnorm_rows(
        _want(out, "out", torch.float32, d), _want(residual, "residual", torch.float32, d),
        _want(add, "add", torch.float32, d), _want(weight, "weight", torch.float32, d), rows, n, eps,
        _stream(residual, stream)))
    return out


def rmsnorm_rope_rows(q: Optional[torch.Tensor], k: Optional[torch.Tensor], wq: Optional[torch.Tensor],
                      wk: Optional[torch.Tensor], cos_table: torch.Tensor, sin_table: torch.Tensor, pos0: int,
                      eps: float, stream: Optional[torch.cuda.Stream] = None) -> None:
    """Per-head RMSNorm + NeoX RoPE in place.  q [T, Hq, D], k [T, Hk, D] (either
    may be None); token t is at position pos0 + t and uses row pos0 + t of the
    [positions, rope_max_dim] cos/sin tables (v7s_rmsnorm_rope_heads on Q then K
    per token, rmsnorm_rope_dispatch.inc:11-52)."""
    shape = _qk_shape(q, k, cos_table, sin_table, pos0)
    if shape is None:
        return
    ref, tokens, head_dim = shape
    d = ref.device
    _check(lib().v7g_rmsnorm_rope_rows(
        _want(q, "q", torch.float32, d), _want(k, "k", torch.float32, d), tokens,
        q.shape[1] if q is not None else 0, k.shape[1] if k is not None else 0, head_dim,
        _want(wq, "wq", torch.float32, d), _want(wk, "wk", torch.float32, d),
        _want(cos_table, "cos_table", torch.float32, d), _want(sin_table, "sin_table", torch.float32, d),
        pos0, cos_table.shape[1], eps, _stream(ref, stream)))


def _qk_shape(q: Optional[torch.Tensor], k: Optional[torch.Tensor], cos_table: torch.Tensor,
              sin_table: torch.Tensor, pos0: int):
    ref = q if q is not None else k
    if ref is None:
        return None
    if ref.dim() != 3:
        raise ValueError("q/k must be [tokens, heads, head_dim]")
    tokens, _, head_dim = ref.shape
    for t in (q, k):
        if t is not None and (t.dim() != 3 or t.shape[0] != tokens or t.shape[2] != head_dim):
            raise ValueError("q and k must agree in tokens and head_dim")
    if cos_table.shape != sin_table.shape or cos_table.dim() != 2:
        raise ValueError("cos/sin tables must be equal [positions, rope_max_dim] tensors")
    if tokens and pos0 + tokens > cos_table.shape[0]:
        raise ValueError("cos/sin tables have fewer rows than pos0 + tokens")
    if cos_table.shape[1] < head_dim // 2:
        raise ValueError("cos/sin table rows must hold at least head_dim/2 entries")
    return ref, tokens, head_dim


def rope_only_rows(q: Optional[torch.Tensor], k: Optional[torch.Tensor], cos_table: torch.Tensor,
                   sin_table: torch.Tensor, pos0: int, stream: Optional[torch.cuda.Stream] = None) -> None:
    """NeoX RoPE without the norm, in place (v7s_rope_only_heads on Q then K per
    token, rope_only_kernel.inc:11-53).  Same layout and tables as
    rmsnorm_rope_rows; tokens at position 0 are left untouched."""
    shape = _qk_shape(q, k, cos_table, sin_table, pos0)
    if shape is None:
        return
    ref, tokens, head_dim = shape
    d = ref.device
    _check(lib().v7g_rope_only_rows(
        _want(q, "q", torch.float32, d), _want(k, "k", torch.float32, d), tokens,
        q.shape[1] if q is not None else 0, k.shape[1] if k is not None else 0, head_dim,
        _want(cos_table, "cos_table", torch.float32, d), _want(sin_table, "sin_table", torch.float32, d),
        pos0, cos_table.shape[1], _stream(ref, stream)))


def _scaling_args(scaling: Optional[dict]):
    if not scaling:
        return 0, 0.0, 0.0, 0.0, 0
    return (1, float(scaling["factor"]), float(scaling["high_freq_factor"]), float(scaling["low_freq_factor"]),
            int(scaling["orig_max_pos"]))


def rope_freqs(half: int, base: float, scaling: Optional[dict] = None):
    """freqs[j] = base^(-j/half) (float64, host) as the reference's x87 table
    builder computes them (fused_f32_kernel.inc:117-147); scaling = None or a
    llama3 dict {"factor", "high_freq_factor", "low_freq_factor",
    "orig_max_pos"} (:149-256)."""
    import numpy as np
    f = np.empty(half, np.float64)
    _check(lib().v7g_rope_freqs(f.ctypes.data, half, base, *_scaling_args(scaling)))
    return f


def rope_tables(positions: int, half: int, base: float, stride: Optional[int] = None, pos0: int = 0,
                scaling: Optional[dict] = None, device: Optional[torch.device] = None,
                stream: Optional[torch.cuda.Stream] = None):
    """cos, sin [positions, stride] fp32 on the device for positions
    pos0..pos0+positions-1: the reference's x87 tables, computed by the
    library's table kernel (columns half.. zero)."""
    import numpy as np
    stride = stride or half
    device = device or torch.device("cuda", torch.cuda.current_device())
    freqs = np.ascontiguousarray(rope_freqs(half, base, scaling))
    cos = torch.empty(positions, stride, dtype=torch.float32, device=device)
    sin = torch.empty_like(cos)
    _check(lib().v7g_rope_tables(_want(cos, "cos", torch.float32, device), _want(sin, "sin", torch.float32, device),
                                 pos0, positions, half, stride, freqs.ctypes.data, _stream(cos, stream)))
    return cos, sin


class _DeviceView:
    """A __cuda_array_interface__ view of library-owned device memory."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": shape, "typestr": typestr, "version": 3,
                                         "strides": None}


def rope_init(head_dim: int, base: float, scaling: Optional[dict] = None):
    """Builds the library's own RoPE tables [ROPE_TABLE_POSITIONS, head_dim/2]
    on the current device (what v7s_rope_init does from the key store) and
    returns (cos, sin) tensors viewing them; the library owns the memory
    until v7s_shutdown or the next rope_init with another head size."""
    L = lib()
    _check(L.v7g_rope_init(head_dim, base, *_scaling_args(scaling)))
    c, s, h = c_void_p(), c_void_p(), c_int()
    _check(L.v7g_get_rope_tables(ctypes.byref(c), ctypes.byref(s), ctypes.byref(h)))
    shape = (ROPE_TABLE_POSITIONS, h.value)
    dev = torch.device("cuda", torch.cuda.current_device())
    return (torch.as_tensor(_DeviceView(c.value, shape, "<f4"), device=dev),
            torch.as_tensor(_DeviceView(s.value, shape, "<f4"), device=dev))


def swiglu(out: torch.Tensor, gate: torch.Tensor, up: torch.Tensor,
           stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """out = (sigmoid(gate) * gate) * up elementwise with v7's sigmoid
    (EVAL_SIGMOID, v7_macros.inc:98-160)."""
    d = gate.device
    if out.shape != gate.shape or up.shape != gate.shape:
        raise ValueError("shape mismatch")
    _check(lib().v7g_swiglu(_want(out, "out", torch.float32, d), _want(gate, "gate", torch.float32, d),
                            _want(up, "up", torch.float32, d), gate.numel(), _stream(gate, stream)))
    return out


def swiglu_q8_rows(codes: torch.Tensor, scales: torch.Tensor, gate: torch.Tensor, up: torch.Tensor,
                   stream: Optional[torch.cuda.Stream] = None) -> None:
    """SwiGLU then Q8 per row: codes [.., n] int8, scales [.., n/64] fp32."""
    rows, n = _rows(gate)
    d = gate.device
    if up.shape != gate.shape or codes.shape != gate.shape or scales.numel() != rows * (n // 64):
        raise ValueError("shape mismatch")
    _check(lib().v7g_swiglu_q8_rows(_want(codes, "codes", torch.int8, d), _want(scales, "scales", torch.float32, d),
                                    _want(gate, "gate", torch.float32, d), _want(up, "up", torch.float32, d),
                                    rows, n, _stream(gate, stream)))


def quantize_rows(codes: torch.Tensor, scales: torch.Tensor, x: torch.Tensor,
                  stream: Optional[torch.cuda.Stream] = None) -> None:
    """Q8 per row (v7d_quantize, utility_dispatch.inc:110-213): codes [.., n] int8,
    scales [.., ceil(n/64)] fp32."""
    rows, n = _rows(x)
    d = x.device
    if codes.shape != x.shape or scales.numel() != rows * ((n + 63) // 64):
        raise ValueError("shape mismatch")
    _check(lib().v7g_quantize_rows(_want(codes, "codes", torch.int8, d), _want(scales, "scales", torch.float32, d),
                                   _want(x, "x", torch.float32, d), rows, n, _stream(x, stream)))


def add_inplace(x: torch.Tensor, y: torch.Tensor, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """x += y (v7s_add_inplace, add_kernel.inc:26-49)."""
    d = x.device
    if x.shape != y.shape:
        raise ValueError("shape mismatch")
    _check(lib().v7g_add_inplace(_want(x, "x", torch.float32, d), _want(y, "y", torch.float32, d), x.numel(),
                                 _stream(x, stream)))
    return x


def rmsnorm_quantize_rows(codes: torch.Tensor, scales: torch.Tensor, x: torch.Tensor, weight: torch.Tensor,
                          eps: float, stream: Optional[torch.cuda.Stream] = None) -> None:
    """RMSNorm then Q8 per row (v7s_rmsnorm_quantize, rmsnorm_quantize_kernel.inc:60-218)."""
    rows, n = _rows(x)
    d = x.device
    if codes.shape != x.shape or scales.numel() != rows * (n // 64) or weight.numel() != n:
        raise ValueError("shape mismatch")
    _check(lib().v7g_rmsnorm_quantize_rows(
        _want(codes, "codes", torch.int8, d), _want(scales, "scales", torch.float32, d),
        _want(x, "x", torch.float32, d), _want(weight, "weight", torch.float32, d), rows, n, eps,
        _stream(x, stream)))


def _gemv_dims(x: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor, out: torch.Tensor):
    if x.dim() != 2 or wq.dim() != 2:
        raise ValueError("activations must be [batch, n], weight codes [d, n]")
    batch, n = x.shape
    d = wq.shape[0]
    if wq.shape[1] != n or ws.numel() != d * (n // 64) or out.shape != (batch, d):
        raise ValueError("shape mismatch: weights [d, n] + [d, n/64] scales, out [batch, d]")
    return batch, n, d


def q8_gemv(out: torch.Tensor, xq: torch.Tensor, xs: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor,
            stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """out[b, i] = dot(x_b, w_i), Q8 activation (codes [batch, n], scales
    [batch, n/64]) times Q8 weights (codes [d, n], scales [d, n/64]) -- v7d_q8
    (q8_kernel.inc:84-207)."""
    batch, n, d = _gemv_dims(xq, wq, ws, out)
    dv = xq.device
    _check(lib().v7g_q8_gemv(_want(out, "out", torch.float32, dv), _want(xq, "xq", torch.int8, dv),
                             _want(xs, "xs", torch.float32, dv), _want(wq, "wq", torch.int8, dv),
                             _want(ws, "ws", torch.float32, dv), batch, n, d, _stream(xq, stream)))
    return out


def q8_fused_gemv(out: torch.Tensor, x: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor,
                  stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """v7d_q8_fused (fused_dispatch.inc:82-114): quantise each fp32 activation
    row with v7d_quantize's rules, then v7d_q8, in one kernel."""
    batch, n, d = _gemv_dims(x, wq, ws, out)
    dv = x.device
    _check(lib().v7g_q8_fused_gemv(_want(out, "out", torch.float32, dv), _want(x, "x", torch.float32, dv),
                                   _want(wq, "wq", torch.int8, dv), _want(ws, "ws", torch.float32, dv), batch, n, d,
                                   _stream(x, stream)))
    return out


def swiglu_q8_gemv(out: torch.Tensor, xq: torch.Tensor, xs: torch.Tensor, gate_q: torch.Tensor, gate_s: torch.Tensor,
                   up_q: torch.Tensor, up_s: torch.Tensor, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """v7d_swiglu_q8 (swiglu_q8_kernel.inc:16-286): out[b, i] =
    swiglu(dot(x_b, gate_i), dot(x_b, up_i)) with a Q8 activation."""
    batch, n, d = _gemv_dims(xq, gate_q, gate_s, out)
    if up_q.shape != gate_q.shape or up_s.numel() != gate_s.numel():
        raise ValueError("gate and up weights must have the same shape")
    dv = xq.device
    _check(lib().v7g_swiglu_q8_gemv(
        _want(out, "out", torch.float32, dv), _want(xq, "xq", torch.int8, dv), _want(xs, "xs", torch.float32, dv),
        _want(gate_q, "gate_q", torch.int8, dv), _want(gate_s, "gate_s", torch.float32, dv),
        _want(up_q, "up_q", torch.int8, dv), _want(up_s, "up_s", torch.float32, dv), batch, n, d, _stream(xq, stream)))
    return out


def swiglu_f32q8_gemv(out: torch.Tensor, x: torch.Tensor, gate_q: torch.Tensor, gate_s: torch.Tensor,
                      up_q: torch.Tensor, up_s: torch.Tensor, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """v7d_swiglu (swiglu_kernel.inc): fp32 activation times Q8 gate/up, SwiGLU
    epilogue, with the reference's dual-row arithmetic."""
    batch, n, d = _gemv_dims(x, gate_q, gate_s, out)
    if up_q.shape != gate_q.shape or up_s.numel() != gate_s.numel():
        raise ValueError("gate and up weights must have the same shape")
    dv = x.device
    _check(lib().v7g_swiglu_f32q8_gemv(
        _want(out, "out", torch.float32, dv), _want(x, "x", torch.float32, dv),
        _want(gate_q, "gate_q", torch.int8, dv), _want(gate_s, "gate_s", torch.float32, dv),
        _want(up_q, "up_q", torch.int8, dv), _want(up_s, "up_s", torch.float32, dv), batch, n, d, _stream(x, stream)))
    return out


def rmsnorm_rows_noalloc(out, x, weight, eps: float, stream: Optional[torch.cuda.Stream] = None):
    """rmsnorm_rows for callers that must not have the library allocate
    device memory: host numpy arrays (or any memory the GPU can address) go
    through a static device array of NOALLOC_SCRATCH_BYTES per GPU, so the
    call never reaches cudaMalloc.  Synchronous; raises V7GError when
    gamma + x + out do not fit in the array."""
    import numpy as np
    for name, a in (("out", out), ("x", x), ("weight", weight)):
        if not isinstance(a, np.ndarray) or a.dtype != np.float32 or not a.flags.c_contiguous:
            raise TypeError(f"{name} must be a C-contiguous float32 numpy array")
    if x.ndim != 2 or out.shape != x.shape or weight.size != x.shape[1]:
        raise ValueError("shape mismatch: x and out [rows, n], weight [n]")
    s = stream.cuda_stream if stream is not None else None
    _check(lib().v7g_rmsnorm_rows_noalloc(out.ctypes.data, x.ctypes.data, weight.ctypes.data, x.shape[0], x.shape[1],
                                          eps, s))
    return out


def fill_normal(dst: torch.Tensor, seed: int, mean: float, std: float, row0: int = 0,
                stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """Deterministic N(mean, std) fill keyed by (seed, row0 + row, col): any row
    shard of a larger matrix is reproducible on its own."""
    rows, n = _rows(dst)
    _check(lib().v7g_fill_normal(_want(dst, "dst", torch.float32, dst.device), rows, n, row0, seed, mean, std,
                                 _stream(dst, stream)))
    return dst


# ------------------------------------------- per-vector, reference-named ops


def set_rms_eps(eps: float) -> None:
    """RMS epsilon used by the reference-named ops (the reference's g_rms_eps)."""
    lib().v7g_set_rms_eps(eps)


def get_rms_eps() -> float:
    return float(lib().v7g_get_rms_eps())


def v7s_rmsnorm(o: torch.Tensor, x: torch.Tensor, weight: torch.Tensor) -> None:
    """src/v7_lib.h:270 -- one vector, size = x.numel() (contract size % 32 == 0)."""
    rmsnorm_rows(o.view(1, -1), x.view(1, -1), weight, get_rms_eps())


def v7s_add_inplace(x: torch.Tensor, y: torch.Tensor) -> None:
    """src/v7_lib.h:271."""
    add_inplace(x, y)


def v7s_fused_add_rmsnorm(o: torch.Tensor, residual: torch.Tensor, add: torch.Tensor, weight: torch.Tensor) -> None:
    """src/v7_lib.h:272."""
    fused_add_rmsnorm_rows(o.view(1, -1), residual.view(1, -1), add.view(1, -1), weight, get_rms_eps())


def v7s_rmsnorm_rope_heads(buf: torch.Tensor, n_heads: int, head_dim: int, norm_weight: torch.Tensor,
                           cos_table: torch.Tensor, sin_table: torch.Tensor, pos: int, rope_max_dim: int) -> None:
    """src/v7_lib.h:273 -- one token's n_heads heads at position pos; the tables
    are flat with rows of rope_max_dim floats."""
    ct = cos_table.view(-1, rope_max_dim)
    st = sin_table.view(-1, rope_max_dim)
    d = buf.device
    _check(lib().v7g_rmsnorm_rope_rows(
        _want(buf, "buf", torch.float32, d), 0, 1, n_heads, 0, head_dim, _want(norm_weight, "norm_weight", torch.float32, d),
        0, _want(ct, "cos_table", torch.float32, d), _want(st, "sin_table", torch.float32, d), pos, rope_max_dim,
        get_rms_eps(), _stream(buf, None)))


def v7s_rope_only_heads(buf: torch.Tensor, n_heads: int, head_dim: int, cos_table: torch.Tensor,
                        sin_table: torch.Tensor, pos: int, rope_max_dim: int) -> None:
    """rope_only_dispatch.inc:10-47 -- one token's n_heads heads at position pos."""
    ct = cos_table.view(-1, rope_max_dim)
    st = sin_table.view(-1, rope_max_dim)
    d = buf.device
    _check(lib().v7g_rope_only_rows(
        _want(buf, "buf", torch.float32, d), 0, 1, n_heads, 0, head_dim, _want(ct, "cos_table", torch.float32, d),
        _want(st, "sin_table", torch.float32, d), pos, rope_max_dim, _stream(buf, None)))


def v7d_quantize(out_q: torch.Tensor, in_x: torch.Tensor, out_s: torch.Tensor) -> None:
    """src/v7_lib.h:123 -- one vector of n = in_x.numel() floats."""
    quantize_rows(out_q.view(1, -1), out_s.view(1, -1), in_x.view(1, -1))


def v7s_rmsnorm_quantize(out_q: torch.Tensor, in_x: torch.Tensor, out_s: torch.Tensor, weight: torch.Tensor) -> None:
    """src/v7_lib.h:124 -- one vector (contract n % 64 == 0)."""
    rmsnorm_quantize_rows(out_q.view(1, -1), out_s.view(1, -1), in_x.view(1, -1), weight, get_rms_eps())


def selftest_arith(device: Optional[torch.device] = None) -> list[int]:
    """Runs the library's exhaustive device check of its fast arithmetic and
    returns the mismatch count of each of its seven tests (all 0 when exact)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    counts = torch.zeros(7, dtype=torch.int64, device=device)
    _check(lib().v7g_selftest_arith(counts.data_ptr(), _stream(counts, None)))
    return [int(c) for c in counts.cpu().tolist()]


def pipeline_timeouts() -> int:
    """Bounded waits of the pipelined kernels that gave up (0 when healthy)."""
    return int(lib().v7g_pipeline_timeouts())


def launch_count() -> int:
    """Kernels launched by the library so far in this process."""
    return int(lib().v7g_launch_count())


def set_launch_overlap(on: bool) -> None:
    """Launch overlap (programmatic dependent launch; on by default): each
    kernel may be scheduled while the kernel ahead of it in the stream drains
    and waits on the device for it before touching memory.  Off: plain
    launches.  Results are the same either way."""
    lib().v7g_set_launch_overlap(1 if on else 0)


def launch_overlap() -> bool:
    return bool(lib().v7g_get_launch_overlap())


def version() -> str:
    return lib().v7g_version().decode()
