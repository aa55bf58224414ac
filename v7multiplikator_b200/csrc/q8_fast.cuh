// q8_fast.cuh -- packed / cheaper forms of the SiLU and Q8 steps in q8.cuh.
// Same operations in the same order on the same values, so the results are
// bit-identical; v7g_selftest_arith checks each against its q8.cuh original
// over every input it can receive.  FTZ compilation units only (arith.cuh).
#pragma once
#include "arith.cuh"
#include "q8.cuh"

namespace v7g {

// v7_sigmoid of two elements: pair arithmetic, Markstein reciprocal.  The
// reciprocal argument d = 1 + 2^i * P(f) lies in [1, 2^117).
__device__ __forceinline__ float2 v7_sigmoid_x2(float g0, float g1)
{
	const float c5 = __uint_as_float(0x3AADD303u), c4 = __uint_as_float(0x3C1E7411u), c3 = __uint_as_float(0x3D635B9Bu),
	            c2 = __uint_as_float(0x3E75FCE0u), c1 = __uint_as_float(0x3F317215u);
	const float2 t = make_float2(fminf(fmaxf(-g0, -80.0f), 80.0f), fminf(fmaxf(-g1, -80.0f), 80.0f));
	const float2 fx = mul2(t, splat2(1.4426950408889634f));
	const float2 big = add2(fx, splat2(kRoundMagic)); // rounds fx to an integer
	// f = fx - (big - magic), written as fx + (big - magic) * -1 (both exact):
	// this is the form the exhaustive checks pass in the compiled kernels; the
	// packed subtraction fx - (big - magic) produced different results on
	// about a quarter of all inputs on sm_100a with CUDA 12.9
	const float2 f = add2(fx, mul2(add2(big, splat2(-kRoundMagic)), splat2(-1.0f)));
	float2 p = fma2(splat2(c5), f, splat2(c4));
	p = fma2(p, f, splat2(c3));
	p = fma2(p, f, splat2(c2));
	p = fma2(p, f, splat2(c1));
	p = fma2(p, f, splat2(1.0f));
	// e = 2^i * p with i = bits(big) - bits(magic) by adding i to p's exponent
	// field: the magic's low 9 bits are zero, so i << 23 is bits(big) << 23
	// modulo 2^32.  Exact, and equal to the reference's multiply by the
	// constructed 2^i: p = P(f) lies in [0.70, 1.42] for |f| <= 1/2 and
	// |i| <= 116 after the clamp, so 2^i * p is a normal float, which the
	// product computes without rounding.
	const float2 e = make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(big.x) << 23)),
	                             __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(big.y) << 23)));
	return rcp_nr2(add2(e, splat2(1.0f)));
}

// (sig * g) * u for two elements.
__device__ __forceinline__ float2 v7_swiglu_x2(float g0, float g1, float u0, float u1)
{
	return mul2(mul2(v7_sigmoid_x2(g0, g1), make_float2(g0, g1)), make_float2(u0, u1));
}

__device__ __forceinline__ float4 v7_swiglu4(float4 g, float4 u)
{
	const float2 a = v7_swiglu_x2(g.x, g.y, u.x, u.y);
	const float2 b = v7_swiglu_x2(g.z, g.w, u.z, u.w);
	return make_float4(a.x, a.y, b.x, b.y);
}

// q8_scale for a finite maximum without the general divide, in single
// precision: wmax / 127 as a product by the constant 1/127 held as two floats,
// Ch + Cl (Ch = RN(1/127), Cl = RN(1/127 - Ch)), evaluated the way Brisebarre
// and Muller give for correctly rounded multiplication by an arbitrary
// precision constant ("Correctly rounded multiplication by arbitrary precision
// constants", IEEE Trans. Computers 57(2), 2008): u = RN(w * Cl), then
// RN(w * Ch + u) in one fused multiply-add.  For this constant that is the
// correctly rounded quotient for every w in the floored range; below 2^-60
// the maximum is first scaled by 2^64 (exactly) so that w * Cl stays a normal
// float under FTZ, and the quotient (at least FLT_MIN, so normal) scaled back
// exactly.  No double-precision instruction: those are a scarce pipe here.
// The reciprocal takes the Markstein form.  An inf or a NaN that survived the
// tree takes the IEEE instructions.  v7g_selftest_arith checks scale and
// reciprocal against div.rn / rcp.rn for every possible maximum.
constexpr float kInv127Hi = 7.87401572e-03f; // 0x3C010204
constexpr float kInv127Lo = 2.93329942e-11f; // 0x2E010204

// The IEEE instructions for an inf or NaN maximum, out of line (rare).
static __device__ __noinline__ float2 q8_scale_ieee(float wmax)
{
	float scale, recip;
	q8_scale(wmax, scale, recip);
	return make_float2(scale, recip);
}

__device__ __forceinline__ void q8_scale_fast(float wmax, float &scale, float &recip)
{
	wmax = x86_max(wmax, kQ8WmaxFloor);
	if (wmax <= 3.402823466e38f) {
		using M = F<true>;
		const bool tiny = wmax < 8.67361738e-19f; // 2^-60
		const float w = tiny ? M::mul(wmax, 1.84467441e19f) : wmax; // * 2^64
		const float q = M::fma(w, kInv127Hi, M::mul(w, kInv127Lo));
		scale = tiny ? M::mul(q, 5.42101086e-20f) : q; // * 2^-64
		recip = rcp_nr(scale); // scale in [FLT_MIN, FLT_MAX/127]: reciprocal normal
	} else {
		const float2 sr = q8_scale_ieee(wmax);
		scale = sr.x;
		recip = sr.y;
	}
}

// q8_scale_fast of two finite maxima (two groups) in pair arithmetic: the
// floor, the two-float product by 1/127 with the 2^64 rescaling of tiny
// maxima, and the Markstein reciprocal, each component the same operations in
// the same order as q8_scale_fast.  The product by the low constant feeds the
// pair multiply-add only as its addend, so no contraction can remove its
// rounding.  Checked against q8_scale for every finite maximum by
// v7g_selftest_arith.
__device__ __forceinline__ void q8_scale_finite2(float w0, float w1, float2 &scale, float2 &recip)
{
	w0 = fmaxf(w0, kQ8WmaxFloor); // no NaN here: fmaxf is MAXPS
	w1 = fmaxf(w1, kQ8WmaxFloor);
	const bool t0 = w0 < 8.67361738e-19f, t1 = w1 < 8.67361738e-19f; // 2^-60
	const float2 big = mul2(make_float2(w0, w1), splat2(1.84467441e19f)); // * 2^64
	const float2 w = make_float2(t0 ? big.x : w0, t1 ? big.y : w1);
	const float2 q = fma2(w, splat2(kInv127Hi), mul2(w, splat2(kInv127Lo)));
	const float2 back = mul2(q, splat2(5.42101086e-20f)); // * 2^-64
	scale = make_float2(t0 ? back.x : q.x, t1 ? back.y : q.y);
	recip = rcp_nr2(scale);
}

// Codes of four values whose products p = h * recip satisfy |p| < 127.5 (a
// group with neither NaN nor infinity, quantised with its own scale: |p| is
// at most 127 (1 + 3 * 2^-24)): the rounded product plus 1.5 * 2^23, whose
// low byte is then the product rounded to the nearest integer, ties to even
// (CVTPS2DQ's rounding; the constant is even, so the adder's tie rule is the
// conversion's).  For such p the reference's saturating packs and -127 floor
// change nothing, so no clamp or range test is needed.  The product and the
// sum are single mul.rn / add.rn instructions: PTX does not contract an
// instruction with an explicit rounding modifier into a fused multiply-add,
// which would skip the product's rounding and move exact ties (the packed
// intrinsics were fused that way in some kernels).  Two full-rate
// instructions per code instead of a multiply and a float-to-int conversion
// (16 results per clock per SM in CUDA's throughput table, against 128 for
// a multiply or an add).
// Checked against q8_code_bits over every such p, and on products next to a
// tie under non-trivial reciprocals, by v7g_selftest_arith.
__device__ __forceinline__ uint32_t q8_codes4_small(float4 h, float recip)
{
	using M = F<true>;
	return pack4_low_bytes(__float_as_uint(M::add(M::mul(h.x, recip), kRoundMagic)),
	                       __float_as_uint(M::add(M::mul(h.y, recip), kRoundMagic)),
	                       __float_as_uint(M::add(M::mul(h.z, recip), kRoundMagic)),
	                       __float_as_uint(M::add(M::mul(h.w, recip), kRoundMagic)));
}

// q8_codes4 with pair arithmetic.
__device__ __forceinline__ uint32_t q8_codes4_x2(float4 h, float recip)
{
	const float2 p01 = mul2(make_float2(h.x, h.y), splat2(recip));
	const float2 p23 = mul2(make_float2(h.z, h.w), splat2(recip));
	const float2 m = splat2(kRoundMagic);
	const float2 b01 = add2(make_float2(fminf(fmaxf(p01.x, -127.0f), 127.0f), fminf(fmaxf(p01.y, -127.0f), 127.0f)), m);
	const float2 b23 = add2(make_float2(fminf(fmaxf(p23.x, -127.0f), 127.0f), fminf(fmaxf(p23.y, -127.0f), 127.0f)), m);
	const uint32_t q0 = fabsf(p01.x) < 2147483648.0f ? __float_as_uint(b01.x) : 0x81u;
	const uint32_t q1 = fabsf(p01.y) < 2147483648.0f ? __float_as_uint(b01.y) : 0x81u;
	const uint32_t q2 = fabsf(p23.x) < 2147483648.0f ? __float_as_uint(b23.x) : 0x81u;
	const uint32_t q3 = fabsf(p23.y) < 2147483648.0f ? __float_as_uint(b23.y) : 0x81u;
	return pack4_low_bytes(q0, q1, q2, q3);
}

// Q8 of U groups held one per half-warp (lane L of a half: elements 4L..4L+3
// of its group as one float4), every group with the reference's rules: codes
// (one word per lane, four codes) and scales.  One vote decides for all of
// the warp's groups whether any holds an infinity or a NaN; when none does,
// the maxima are plain integer maxima of the magnitudes, the scales come in
// pair arithmetic and each code from one rounded product and one rounded sum
// (|h * recip| < 127.5 there, so the reference's saturation never acts);
// otherwise the general path runs: the exact MAXPS tree (a NaN makes the
// order matter), the IEEE scale for an infinite maximum, clamped codes.
// Must be called by all 32 lanes.
template <int U>
__device__ __forceinline__ void q8_groups_f4(const float4 (&h)[U], int lane, uint32_t (&code)[U], float (&scale)[U])
{
	uint32_t m[U];
#pragma unroll
	for (int u = 0; u < U; ++u)
		m[u] = max(max(abs_bits(h[u].x), abs_bits(h[u].y)), max(abs_bits(h[u].z), abs_bits(h[u].w)));
#pragma unroll
	for (int mask = 1; mask <= 8; mask <<= 1)
#pragma unroll
		for (int u = 0; u < U; ++u)
			m[u] = max(m[u], __shfl_xor_sync(kFullMask, m[u], mask));
	bool special = false;
#pragma unroll
	for (int u = 0; u < U; ++u)
		special |= m[u] >= 0x7f800000u;
	if (!__any_sync(kFullMask, special)) {
#pragma unroll
		for (int u = 0; u < U; u += 2) {
			float2 sc, rc;
			q8_scale_finite2(__uint_as_float(m[u]), __uint_as_float(m[u + 1 < U ? u + 1 : u]), sc, rc);
			scale[u] = sc.x;
			code[u] = q8_codes4_small(h[u], rc.x);
			if (u + 1 < U) {
				scale[u + 1] = sc.y;
				code[u + 1] = q8_codes4_small(h[u + 1], rc.y);
			}
		}
	} else {
		// rare (an infinity or NaN in the warp's groups)
#pragma unroll
		for (int u = 0; u < U; ++u) {
			float recip;
			q8_scale_fast(group_absmax_f4(h[u], lane), scale[u], recip);
			code[u] = q8_codes4_x2(h[u], recip);
		}
	}
}

} // namespace v7g
