// arith.cuh -- packed fp32 pairs and a cheap correctly rounded reciprocal for
// the streaming SwiGLU and Q8 kernels.
//
// sm_100 executes fp32 add/mul/fma on two lanes of a register pair in one
// instruction (CUDA's __fadd2_rn / __fmul2_rn / __ffma2_rn); each component is
// an ordinary IEEE operation with its own rounding, so a pair computes exactly
// what two scalar instructions compute, in half the issue slots.  The
// reference runs these kernels with FTZ+DAZ; the intrinsics follow the
// compilation unit's -ftz setting, so this header may only be used from units
// built with -ftz=true (build.py defines V7G_FTZ_TU for them).
//
// A pair product that feeds a pair sum directly can come out fused into one
// multiply-add in some kernels (seen with a product added to a rounding
// constant), losing the product's rounding.  Code that relies on that
// rounding must not have that shape: q8_codes4_small uses scalar mul.rn and
// add.rn in inline PTX, which PTX never contracts; the other kernels put a separate step between
// (q8_codes4_x2 its clamp) or use the product more than once (v7_sigmoid_x2),
// and v7g_selftest_arith checks each over its inputs.  (Inline-PTX pair
// operations would rule it out but cost a third of the SwiGLU throughput in
// register-pair moves.)
//
// rcp.rn expands to a general sequence with special-case branches.  For the
// arguments these kernels have (finite, normal, normal reciprocal) the
// correctly rounded 1/d comes from the hardware reciprocal seed (rcp.approx,
// at most 1 ulp off, PTX ISA) and one Newton-Raphson correction in
// Markstein's form (P. Markstein, "Computation of elementary functions on the
// IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990): the
// residual r = 1 - d*y in one fused multiply-add, then y + y*r rounded once.
// v7g_selftest_arith checks it against rcp.rn for every normal d whose
// reciprocal is normal, scalar and packed.
#pragma once
#include <cstdint>

#include "fp.cuh"

#ifndef V7G_FTZ_TU
#error "arith.cuh needs a compilation unit built with -ftz=true -DV7G_FTZ_TU"
#endif

namespace v7g {

__device__ __forceinline__ float2 splat2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

__device__ __forceinline__ float rcp_seed(float d)
{
	float y;
	asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(d));
	return y;
}

// 1/d correctly rounded, for finite normal d whose reciprocal is normal.
__device__ __forceinline__ float rcp_nr(float d) { return rcp_nr_ftz(d); }

// The pair form: both corrections in packed instructions.
__device__ __forceinline__ float2 rcp_nr2(float2 d)
{
	const float2 y = make_float2(rcp_seed(d.x), rcp_seed(d.y));
	const float2 r = fma2(make_float2(-d.x, -d.y), y, splat2(1.0f));
	return fma2(y, r, y);
}

} // namespace v7g
