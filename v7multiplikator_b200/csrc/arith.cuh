// arith.cuh -- packed fp32 pairs and the cheap correctly rounded reciprocal /
// divide used by the streaming SwiGLU and Q8 kernels.
//
// sm_100 executes fp32 add/mul/fma on two lanes of a 64-bit register pair in
// one instruction (PTX add/sub/mul/fma .f32x2); each half is an ordinary IEEE
// operation with its own rounding, so a pair computes exactly what two scalar
// instructions compute, in half the issue slots.
//
// The IEEE div.rn / rcp.rn instructions expand to a general sequence with
// special-case branches.  In the ranges these kernels need, the correctly
// rounded results come from the hardware reciprocal seed (rcp.approx: at most
// 1 ulp off, PTX ISA) followed by one Newton-Raphson correction in Markstein's
// form (P. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Dev. 34(1), 1990): the residual
// r = 1 - d*y is exact in one fused multiply-add and y + y*r is rounded once.
// Quotients use the same correction from the correctly rounded reciprocal of
// the divisor.  Both are checked exhaustively against rcp.rn / div.rn over
// every input they receive (v7g_selftest_arith).  All FTZ (the kernels using
// them run with the reference's FTZ+DAZ).
#pragma once
#include <cstdint>

#include "fp.cuh"

namespace v7g {

typedef unsigned long long f32x2;

__device__ __forceinline__ f32x2 pack2(float a, float b)
{
	f32x2 r;
	asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
	return r;
}
__device__ __forceinline__ void unpack2(f32x2 v, float &a, float &b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v)); }
__device__ __forceinline__ f32x2 splat2(float a) { return pack2(a, a); }

__device__ __forceinline__ f32x2 add2(f32x2 a, f32x2 b)
{
	f32x2 r;
	asm("add.rn.ftz.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
	return r;
}
__device__ __forceinline__ f32x2 sub2(f32x2 a, f32x2 b)
{
	f32x2 r;
	asm("sub.rn.ftz.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
	return r;
}
__device__ __forceinline__ f32x2 mul2(f32x2 a, f32x2 b)
{
	f32x2 r;
	asm("mul.rn.ftz.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
	return r;
}
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c)
{
	f32x2 r;
	asm("fma.rn.ftz.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
	return r;
}

__device__ __forceinline__ float rcp_seed(float d)
{
	float y;
	asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(d));
	return y;
}

// 1/d correctly rounded, for finite normal d whose reciprocal is normal.
__device__ __forceinline__ float rcp_nr(float d)
{
	using M = F<true>;
	const float y = rcp_seed(d);
	const float r = M::fma(-d, y, 1.0f);
	return M::fma(y, r, y);
}

// The pair form.  `nd` is -d (the callers produce it for free).
__device__ __forceinline__ f32x2 rcp_nr2(f32x2 d, f32x2 nd)
{
	float d0, d1;
	unpack2(d, d0, d1);
	const f32x2 y = pack2(rcp_seed(d0), rcp_seed(d1));
	const f32x2 r = fma2(nd, y, splat2(1.0f));
	return fma2(y, r, y);
}

// RN(1/127), the divisor of the Q8 scale.
constexpr uint32_t kRcp127Bits = 0x3C010204u;

// a / 127 correctly rounded, for finite a >= 0 whose quotient is normal.
__device__ __forceinline__ float div127(float a)
{
	using M = F<true>;
	const float y = __uint_as_float(kRcp127Bits);
	const float q = M::mul(a, y);
	const float r = M::fma(-127.0f, q, a);
	return M::fma(r, y, q);
}

} // namespace v7g
