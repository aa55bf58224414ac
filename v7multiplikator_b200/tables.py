"""Host-side RoPE table producer.

NeoX half-split rotary tables for the RMSNorm+RoPE kernel: row p, column j
(j < half) holds cos / sin of p * base^(-j/half), computed in double precision
and rounded to fp32; columns half..stride-1 are zero.  This restates the
reference's table builder (fused_f32_kernel.inc:120-147, :257-302, which uses
x87 extended precision) without its optional llama3 frequency scaling.  The
tables are kernel inputs: the same bytes go to the device and to any checker.
"""
from __future__ import annotations

import numpy as np


def rope_tables(positions: int, half: int, stride: int | None = None, base: float = 1e6):
    stride = stride or half
    if half <= 0 or stride < half or positions < 0 or not base > 0:
        raise ValueError("need half > 0, stride >= half, positions >= 0, base > 0")
    j = np.arange(half, dtype=np.float64)
    freq = base ** (-j / half)
    ang = np.arange(positions, dtype=np.float64)[:, None] * freq[None, :]
    cos = np.zeros((positions, stride), np.float32)
    sin = np.zeros((positions, stride), np.float32)
    cos[:, :half] = np.cos(ang)
    sin[:, :half] = np.sin(ang)
    return cos, sin
