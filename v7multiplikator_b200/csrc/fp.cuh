// fp.cuh -- IEEE fp32 operations with explicit rounding and denormal mode.
//
// v7's kernels are defined by their x86 instruction sequence: every vmulps,
// vaddps, vdivss, vsqrtss rounds once, only vfmadd* fuses, and the kernels the
// reference runs on its dispatched worker threads do so with MXCSR FTZ+DAZ set
// (v7_init.inc:103-109).  To reproduce those results bit for bit the device
// code spells every operation as one PTX instruction: the compiler can neither
// contract a multiply-add nor change a rounding, and the .ftz variants give
// the FTZ+DAZ behaviour (subnormal inputs read as zero, subnormal results
// flushed) where the reference has it.
#pragma once
#include <cstdint>

namespace v7g {

template <bool FTZ>
struct F;

#define V7G_FP_BODY(SUF)                                                                                          \
	static __device__ __forceinline__ float add(float a, float b)                                                  \
	{                                                                                                              \
		float r;                                                                                                   \
		asm("add.rn" SUF ".f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));                                           \
		return r;                                                                                                  \
	}                                                                                                              \
	static __device__ __forceinline__ float sub(float a, float b)                                                  \
	{                                                                                                              \
		float r;                                                                                                   \
		asm("sub.rn" SUF ".f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));                                           \
		return r;                                                                                                  \
	}                                                                                                              \
	static __device__ __forceinline__ float mul(float a, float b)                                                  \
	{                                                                                                              \
		float r;                                                                                                   \
		asm("mul.rn" SUF ".f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));                                           \
		return r;                                                                                                  \
	}                                                                                                              \
	static __device__ __forceinline__ float fma(float a, float b, float c)                                         \
	{                                                                                                              \
		float r;                                                                                                   \
		asm("fma.rn" SUF ".f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));                               \
		return r;                                                                                                  \
	}                                                                                                              \
	static __device__ __forceinline__ float div(float a, float b)                                                  \
	{                                                                                                              \
		float r;                                                                                                   \
		asm("div.rn" SUF ".f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));                                           \
		return r;                                                                                                  \
	}                                                                                                              \
	/* correctly rounded 1/a: equal to div(1, a) */                                                                \
	static __device__ __forceinline__ float rcp(float a)                                                           \
	{                                                                                                              \
		float r;                                                                                                   \
		asm("rcp.rn" SUF ".f32 %0, %1;" : "=f"(r) : "f"(a));                                                       \
		return r;                                                                                                  \
	}                                                                                                              \
	static __device__ __forceinline__ float sqrt(float a)                                                          \
	{                                                                                                              \
		float r;                                                                                                   \
		asm("sqrt.rn" SUF ".f32 %0, %1;" : "=f"(r) : "f"(a));                                                      \
		return r;                                                                                                  \
	}

template <>
struct F<false> {
	V7G_FP_BODY("")
};
template <>
struct F<true> {
	V7G_FP_BODY(".ftz")
};
#undef V7G_FP_BODY

// Correctly rounded 1/d under FTZ for normal d with a normal reciprocal: the
// hardware reciprocal seed (rcp.approx, at most 1 ulp off) and one
// Newton-Raphson correction in Markstein's form (P. Markstein, IBM J. Res.
// Dev. 34(1), 1990).  Checked against rcp.rn.ftz for every such d by
// v7g_selftest_arith.
__device__ __forceinline__ float rcp_nr_ftz(float d)
{
	float y;
	asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(d));
	const float r = F<true>::fma(-d, y, 1.0f);
	return F<true>::fma(y, r, y);
}

// x86 MAXPS/MAXSS: the second operand is returned when either input is NaN
// (or both are zero).  MINPS/MINSS likewise.
__device__ __forceinline__ float x86_max(float a, float b) { return a > b ? a : b; }
__device__ __forceinline__ float x86_min(float a, float b) { return a < b ? a : b; }

// 1.5 * 2^23: adding it to |v| < 2^22 rounds v to an integer in the low
// mantissa bits (round to nearest even, the FP adder's own rounding), and
// float_as_int(v + kRoundMagic) - kRoundMagicBits is that integer.
constexpr float kRoundMagic = 12582912.0f;
constexpr int32_t kRoundMagicBits = 0x4B400000;

} // namespace v7g
