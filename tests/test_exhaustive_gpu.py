"""The production kernels against their scalar counterparts over every fp32
input, end to end.

The fast kernels (float4 / packed-pair arithmetic, Markstein reciprocal) and
the general kernels (one plain IEEE instruction per step, checked against the
oracle in test_parity_gpu.py) compute the same function by construction; here
that is verified on the compiled kernels themselves, for all 2^32 bit
patterns of the activation, in chunks of 2^28: gate = the patterns, up = 1.
The general kernels are reached with an output that is not 16-byte
aligned."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
CHUNK = 1 << 28


def patterns(start: int, dev) -> torch.Tensor:
    """2^28 consecutive fp32 bit patterns from `start`, one element of padding
    in front (so [1:] is 4-byte offset)."""
    buf = torch.zeros(CHUNK + 4, dtype=torch.int32, device=dev)
    buf[4:].copy_(torch.arange(start, start + CHUNK, dtype=torch.int64, device=dev).to(torch.int32))
    return buf.view(torch.float32)


def same_bits(a: torch.Tensor, b: torch.Tensor) -> bool:
    nan = torch.isnan(a)
    return bool(torch.equal(nan, torch.isnan(b)) and torch.equal(a.view(torch.int32)[~nan], b.view(torch.int32)[~nan]))


def test_swiglu_fast_equals_scalar_all_inputs(cuda):
    import v7multiplikator_b200 as v7g
    ones = torch.ones(CHUNK + 4, device=cuda)
    out_fast = torch.empty(CHUNK + 4, device=cuda)
    out_ref = torch.empty(CHUNK + 4, device=cuda)
    for c in range(1 << 4):
        g = patterns(c * CHUNK, cuda)
        v7g.swiglu(out_fast[4:], g[4:], ones[4:])           # all 16-byte aligned: float4 / packed kernel
        v7g.swiglu(out_ref[1:CHUNK + 1], g[4:], ones[4:])   # output 4 bytes off: scalar kernel
        torch.cuda.synchronize()
        assert same_bits(out_fast[4:], out_ref[1:CHUNK + 1]), f"chunk {c}"


@pytest.mark.parametrize("swiglu", [True, False], ids=["swiglu_q8", "quantize"])
def test_q8_fast_equals_general_all_inputs(cuda, swiglu):
    import v7multiplikator_b200 as v7g
    n = 1 << 16
    rows = CHUNK // n
    ones = torch.ones(CHUNK + 4, device=cuda)
    codes_fast = torch.empty(CHUNK + 16, dtype=torch.int8, device=cuda)
    codes_ref = torch.empty(CHUNK + 16, dtype=torch.int8, device=cuda)
    s_fast = torch.empty(rows, n // 64, device=cuda)
    s_ref = torch.empty(rows, n // 64, device=cuda)
    for c in range(1 << 4):
        g = patterns(c * CHUNK, cuda)
        # general kernel: codes 1 byte off alignment, same activations
        cf, cr = codes_fast[16:].view(rows, n), codes_ref[1:CHUNK + 1].view(rows, n)
        if swiglu:
            v7g.swiglu_q8_rows(cf, s_fast, g[4:].view(rows, n), ones[4:].view(rows, n))
            v7g.swiglu_q8_rows(cr, s_ref, g[4:].view(rows, n), ones[4:].view(rows, n))
        else:
            v7g.quantize_rows(cf, s_fast, g[4:].view(rows, n))
            v7g.quantize_rows(cr, s_ref, g[4:].view(rows, n))
        torch.cuda.synchronize()
        assert torch.equal(cf, cr), f"codes, chunk {c}"
        assert same_bits(s_fast, s_ref), f"scales, chunk {c}"
