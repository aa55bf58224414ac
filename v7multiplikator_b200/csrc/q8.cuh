// q8.cuh -- v7's Q8 quantiser and SiLU in device code.
//
// Q8 layout (src/q8_batch4.h:15-19, docs/architecture.md:434-442): int8 codes
// row-major, one fp32 absmax scale per 64-element group.  Group rule
// (quantize_kernel.inc:62-106):
//   wmax  = MAXPS tree of |x| over the group, floored at 127 * 2^-126
//   scale = wmax / 127 (exact divide), recip = 1 / scale (exact divide)
//   code  = CVTPS2DQ(x * recip) -> saturating packs -> max(code, -127)
// all under FTZ+DAZ.
#pragma once
#include "fp.cuh"
#include "reduce.cuh"

namespace v7g {

constexpr int kQ8Group = 64;
// 127 * 2^-126: the floor that makes an all-zero group's scale exactly
// FLT_MIN (quantize_kernel.inc:40-41).
constexpr float kQ8WmaxFloor = 1.4928778e-36f;

__device__ __forceinline__ uint32_t abs_bits(float v) { return __float_as_uint(v) & 0x7fffffffu; }

// Code of one element of a full group, as the reference's vector path makes
// it.  For finite |p| < 2^31, rounding then saturating to [-127, 127] equals
// clamping then rounding; NaN and |p| >= 2^31 convert to INT_MIN in CVTPS2DQ,
// which the packs and the -127 floor turn into -127.  Returns the code in the
// low byte of the result (the upper bytes are don't-care).
__device__ __forceinline__ uint32_t q8_code_bits(float p)
{
	float c = fminf(fmaxf(p, -127.0f), 127.0f); // fmaxf(NaN, -127) = -127
	uint32_t bits = __float_as_uint(c + kRoundMagic);
	return fabsf(p) < 2147483648.0f ? bits : 0x81u; // 0x81 = -127
}

// Code of one element of a trailing (< 64) group, the reference's scalar
// path (quantize_kernel.inc:143-152): clamp as floats (NaN -> -127), then
// round.
__device__ __forceinline__ uint32_t q8_tail_code_bits(float p)
{
	p = x86_max(p, -127.0f);
	p = x86_min(p, 127.0f);
	return __float_as_uint(p + kRoundMagic);
}

// Low bytes of four code words packed into one little-endian word.
__device__ __forceinline__ uint32_t pack4_low_bytes(uint32_t a, uint32_t b, uint32_t c, uint32_t d)
{
	uint32_t ab = __byte_perm(a, b, 0x0040);
	uint32_t cd = __byte_perm(c, d, 0x0040);
	return __byte_perm(ab, cd, 0x5410);
}

// Group absmax in the reference's MAXPS order for the float4 layout: a group
// is one half-warp, lane L (0..15 within the half) holding elements 4L..4L+3.
// Element e sits in 8-float block e/8 (lanes 2b, 2b+1) and lane class e%8.
// The reference's tree is: blocks (0,1),(2,3),(4,5),(6,7) -> (01,23),(45,67)
// -> (03,47) per class, then classes j vs j+4, then (0,2),(1,3), then (0,1)
// (quantize_kernel.inc:62-83).  Lane partners: 2, 4, 8, then 1.
__device__ __forceinline__ float group_absmax_f4_tree(float4 h, int lane)
{
	float a0 = fabsf(h.x), a1 = fabsf(h.y), a2 = fabsf(h.z), a3 = fabsf(h.w);
#pragma unroll
	for (int mask = 2; mask <= 8; mask <<= 1) {
		a0 = max_tree_step(a0, mask, lane);
		a1 = max_tree_step(a1, mask, lane);
		a2 = max_tree_step(a2, mask, lane);
		a3 = max_tree_step(a3, mask, lane);
	}
	a0 = max_tree_step(a0, 1, lane);
	a1 = max_tree_step(a1, 1, lane);
	a2 = max_tree_step(a2, 1, lane);
	a3 = max_tree_step(a3, 1, lane);
	float w0 = x86_max(a0, a2);
	float w1 = x86_max(a1, a3);
	return x86_max(w0, w1);
}

// Same result, fast: without NaN every order gives the true maximum, and for
// non-negative floats the maximum is the largest bit pattern.  The exact tree
// runs only when some group of the warp holds a NaN (which makes the result
// depend on where the NaN sits).  Must be called by all 32 lanes.
__device__ __forceinline__ float group_absmax_f4(float4 h, int lane)
{
	uint32_t m = max(max(abs_bits(h.x), abs_bits(h.y)), max(abs_bits(h.z), abs_bits(h.w)));
	m = max(m, __shfl_xor_sync(kFullMask, m, 1));
	m = max(m, __shfl_xor_sync(kFullMask, m, 2));
	m = max(m, __shfl_xor_sync(kFullMask, m, 4));
	m = max(m, __shfl_xor_sync(kFullMask, m, 8));
	if (__any_sync(kFullMask, m > 0x7f800000u))
		return group_absmax_f4_tree(h, lane);
	return __uint_as_float(m);
}

// Scale and reciprocal of a group from its absmax (quantize_kernel.inc:84-88).
__device__ __forceinline__ void q8_scale(float wmax, float &scale, float &recip)
{
	using M = F<true>;
	wmax = x86_max(wmax, kQ8WmaxFloor);
	scale = M::div(wmax, 127.0f);
	recip = M::rcp(scale);
}

// Quantise a float4 of a full group with its reciprocal; returns the four
// codes packed little-endian.
__device__ __forceinline__ uint32_t q8_codes4(float4 h, float recip)
{
	using M = F<true>;
	return pack4_low_bytes(q8_code_bits(M::mul(h.x, recip)), q8_code_bits(M::mul(h.y, recip)),
	                       q8_code_bits(M::mul(h.z, recip)), q8_code_bits(M::mul(h.w, recip)));
}

// EVAL_SIGMOID (v7_macros.inc:98-160) under FTZ+DAZ: 1 / (1 + 2^i * P(f)) with
// -g clamped to [-80, 80], i = rint(-g*log2e), f = -g*log2e - i and P the
// reference's degree-5 polynomial (coefficients math_data.inc:25-34), Horner
// with fused multiply-adds, then an exact reciprocal.
__device__ __forceinline__ float v7_sigmoid(float g)
{
	using M = F<true>;
	const float c5 = __uint_as_float(0x3AADD303u), c4 = __uint_as_float(0x3C1E7411u), c3 = __uint_as_float(0x3D635B9Bu),
	            c2 = __uint_as_float(0x3E75FCE0u), c1 = __uint_as_float(0x3F317215u);
	float t = fminf(fmaxf(-g, -80.0f), 80.0f); // MAXPS/MINPS against the constant: NaN -> -80
	float fx = M::mul(t, 1.4426950408889634f);
	float big = M::add(fx, kRoundMagic);       // round to nearest even integer
	float ip = M::sub(big, kRoundMagic);
	float f = M::sub(fx, ip);
	int32_t ipi = (int32_t)__float_as_uint(big) - kRoundMagicBits;
	float p = M::fma(c5, f, c4);
	p = M::fma(p, f, c3);
	p = M::fma(p, f, c2);
	p = M::fma(p, f, c1);
	p = M::fma(p, f, 1.0f);
	float two_i = __uint_as_float((uint32_t)(ipi + 127) << 23);
	float e = M::mul(two_i, p);
	float d = M::add(e, 1.0f);
	return M::rcp(d);
}

// SwiGLU in the reference's product order (sig * g) * u
// (swiglu_q8_kernel.inc:204-209).
__device__ __forceinline__ float v7_swiglu(float g, float u)
{
	using M = F<true>;
	return M::mul(M::mul(v7_sigmoid(g), g), u);
}


} // namespace v7g

namespace v7g {

// Group absmax in the reference's MAXPS order for the warp layout used by the
// row kernels: a group is one warp, lane l holding element l (blocks 0..3)
// and element 32 + l (blocks 4..7).  Block pairs (0,1),(2,3) are lanes l and
// l^8; (01,23) are l and l^16; the two halves meet in-lane; then classes j vs
// j+4 (l^4), (0,2)/(1,3) (l^2) and (0,1) (l^1).
__device__ __forceinline__ float group_absmax_w2_tree(float h0, float h1, int lane)
{
	float a = fabsf(h0), b = fabsf(h1);
	a = max_tree_step(a, 8, lane);
	b = max_tree_step(b, 8, lane);
	a = max_tree_step(a, 16, lane);
	b = max_tree_step(b, 16, lane);
	float m = x86_max(a, b);
	m = max_tree_step(m, 4, lane);
	m = max_tree_step(m, 2, lane);
	m = max_tree_step(m, 1, lane);
	return m;
}

// Same result with the bit-pattern maximum when no lane holds a NaN.  Must be
// called by all 32 lanes.
__device__ __forceinline__ float group_absmax_w2(float h0, float h1, int lane)
{
	uint32_t m = max(abs_bits(h0), abs_bits(h1));
	m = max(m, __shfl_xor_sync(kFullMask, m, 1));
	m = max(m, __shfl_xor_sync(kFullMask, m, 2));
	m = max(m, __shfl_xor_sync(kFullMask, m, 4));
	m = max(m, __shfl_xor_sync(kFullMask, m, 8));
	m = max(m, __shfl_xor_sync(kFullMask, m, 16));
	if (__any_sync(kFullMask, m > 0x7f800000u))
		return group_absmax_w2_tree(h0, h1, lane);
	return __uint_as_float(m);
}

// Absmax of a trailing group: the scalar path folds |x_i| into the running
// maximum as MAXSS(|x_i|, wmax), which drops a NaN element, so the result is
// the largest non-NaN magnitude (0 when there is none) in any order.
__device__ __forceinline__ float tail_absmax_w2(float h0, bool v0, float h1, bool v1)
{
	uint32_t a = v0 ? abs_bits(h0) : 0u, b = v1 ? abs_bits(h1) : 0u;
	if (a > 0x7f800000u)
		a = 0u;
	if (b > 0x7f800000u)
		b = 0u;
	uint32_t m = max(a, b);
#pragma unroll
	for (int mask = 1; mask < 32; mask <<= 1)
		m = max(m, __shfl_xor_sync(kFullMask, m, mask));
	return __uint_as_float(m);
}

} // namespace v7g
