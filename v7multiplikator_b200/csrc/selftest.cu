// selftest.cu -- exhaustive device check of the fast arithmetic in arith.cuh
// and q8.cuh against the plain IEEE instructions it replaces.
//
//   test 0  rcp_nr(d) == rcp.rn.ftz(d) for every normal d in [2^-126, 2^126)
//   test 1  rcp_nr2 == rcp.rn.ftz on both halves, same range (the halves
//           paired with different mantissas and exponents)
//   test 2  v7_sigmoid_x2 == v7_sigmoid for all 2^32 bit patterns of g
//   test 3  q8_codes4_x2 code == q8_code_bits code for all 2^32 bit patterns
//           of p = h * recip (recip = 1, so p = h)
//   test 4  q8_scale_fast == q8_scale (scale and reciprocal) for every normal
//           absmax in [2^-127, 2^128) plus inf and NaN; q8_scale_finite2 ==
//           q8_scale for every finite absmax, in both halves of the pair
//   test 5  q8_codes4_small code == q8_code_bits code for every p with
//           |p| < 127.5 (recip = 1, so p = h)
//   test 6  q8_codes4_small and q8_codes4_x2 == q8_code_bits
//           of the rounded product h * recip, for 2^31 products within a few
//           ulps of a rounding tie m + 1/2 under 2^16 reciprocals: where the
//           product's own rounding decides the code (a fused multiply-add
//           would not round it)
// The counts of mismatches are the kernel's output (all zero when the fast
// forms are exact over their whole input range).
#include "internal.h"
#include "launch.cuh"
#include "q8_fast.cuh"

namespace v7g {
namespace {

constexpr int kBlock = 256;

__device__ __forceinline__ float from_exp_mant(int e, uint32_t m) { return __uint_as_float(((uint32_t)(e + 127) << 23) | m); }

__global__ void __launch_bounds__(kBlock) k_selftest(unsigned long long *counts)
{
	kernel_entry();
	const uint64_t stride = (uint64_t)gridDim.x * kBlock;
	const uint64_t tid = (uint64_t)blockIdx.x * kBlock + threadIdx.x;
	unsigned long long bad[7] = {0, 0, 0, 0, 0, 0, 0};
	// test 0: exponents -126 .. 125
	for (uint64_t i = tid; i < (252ull << 23); i += stride) {
		const float d = from_exp_mant((int)(i >> 23) - 126, (uint32_t)(i & 0x7fffff));
		bad[0] += __float_as_uint(rcp_nr(d)) != __float_as_uint(F<true>::rcp(d));
	}
	// test 1: same range, the high half walking the space in reverse
	for (uint64_t i = tid; i < (252ull << 23); i += stride) {
		const uint64_t j = (252ull << 23) - 1 - i;
		const float d0 = from_exp_mant((int)(i >> 23) - 126, (uint32_t)(i & 0x7fffff));
		const float d1 = from_exp_mant((int)(j >> 23) - 126, (uint32_t)((j * 2654435761ull) & 0x7fffff));
		const float2 y = rcp_nr2(make_float2(d0, d1));
		bad[1] += (__float_as_uint(y.x) != __float_as_uint(F<true>::rcp(d0))) + (__float_as_uint(y.y) != __float_as_uint(F<true>::rcp(d1)));
	}
	// tests 2 and 3: every 32-bit pattern, two per thread step
	for (uint64_t i = tid; i < (1ull << 31); i += stride) {
		const float g0 = __uint_as_float((uint32_t)(2 * i)), g1 = __uint_as_float((uint32_t)(2 * i + 1));
		const float2 s = v7_sigmoid_x2(g0, g1);
		bad[2] += (__float_as_uint(s.x) != __float_as_uint(v7_sigmoid(g0))) + (__float_as_uint(s.y) != __float_as_uint(v7_sigmoid(g1)));
		const uint32_t packed = q8_codes4_x2(make_float4(g0, g1, g0, g1), 1.0f);
		const uint32_t want = pack4_low_bytes(q8_code_bits(g0), q8_code_bits(g1), q8_code_bits(g0), q8_code_bits(g1));
		bad[3] += packed != want;
	}
	// test 4: exponents -127 (subnormal range read as zero under FTZ) .. 127, then inf, NaN
	for (uint64_t i = tid; i < (255ull << 23) + 2; i += stride) {
		float w;
		if (i < (255ull << 23))
			w = i < (1ull << 23) ? __uint_as_float((uint32_t)i) : from_exp_mant((int)(i >> 23) - 127, (uint32_t)(i & 0x7fffff));
		else
			w = i == (255ull << 23) ? __int_as_float(0x7f800000) : __int_as_float(0x7fc00000);
		float s_fast, r_fast, s_ref, r_ref;
		q8_scale_fast(w, s_fast, r_fast);
		q8_scale(w, s_ref, r_ref);
		const bool same_s = __float_as_uint(s_fast) == __float_as_uint(s_ref) || (s_fast != s_fast && s_ref != s_ref);
		const bool same_r = __float_as_uint(r_fast) == __float_as_uint(r_ref) || (r_fast != r_fast && r_ref != r_ref);
		bad[4] += !(same_s && same_r);
		// the pair form, for every finite maximum, in either half of the pair
		if (w <= 3.402823466e38f) {
			const float w2 = __uint_as_float(__float_as_uint(w) ^ ((uint32_t)i * 2654435761u & 0x007fffffu));
			float s2_ref, r2_ref;
			q8_scale(w2, s2_ref, r2_ref);
			float2 s2, r2;
			q8_scale_finite2(w, w2, s2, r2);
			bad[4] += (__float_as_uint(s2.x) != __float_as_uint(s_ref)) + (__float_as_uint(r2.x) != __float_as_uint(r_ref)) +
			          (__float_as_uint(s2.y) != __float_as_uint(s2_ref)) + (__float_as_uint(r2.y) != __float_as_uint(r2_ref));
		}
	}
	// test 5: magnitudes below 127.5 (bit patterns up to 0x42FEFFFF), both signs
	for (uint64_t i = tid; i < 0x42ff0000ull; i += stride) {
		const float p0 = __uint_as_float((uint32_t)i), p1 = __uint_as_float((uint32_t)i | 0x80000000u);
		const uint32_t packed = q8_codes4_small(make_float4(p0, p1, p1, p0), 1.0f);
		const uint32_t want = pack4_low_bytes(q8_code_bits(p0), q8_code_bits(p1), q8_code_bits(p1), q8_code_bits(p0));
		bad[5] += packed != want;
	}
	// test 6: i = [recip 16 bits | tie 8 bits | offset 7 bits]; recip in
	// [2^-7, 2^9) spread over mantissas and exponents, h = RN(t / recip)
	// nudged by -3..+3 ulps, t = m + 1/2 for m in [-128, 127]
	for (uint64_t i = tid; i < (1ull << 31); i += stride) {
		const uint32_t ri = (uint32_t)(i >> 15);
		const float recip = from_exp_mant((int)(ri >> 12) - 7, (ri * 2654435761u) & 0x7fffffu);
		const float t = (float)((int)((i >> 7) & 0xff) - 128) + 0.5f;
		const int nudge = (int)(i & 7) - 3;
		const float h0 = F<true>::div(t, recip);
		const float h = __uint_as_float(__float_as_uint(h0) + nudge);
		const float p = F<true>::mul(h, recip);
		const uint32_t want = q8_code_bits(p) & 0xffu;
		const float4 h4 = make_float4(h, h, h, h);
		const uint32_t small = fabsf(p) < 127.5f ? q8_codes4_small(h4, recip) : want * 0x01010101u;
		const uint32_t x2 = q8_codes4_x2(h4, recip);
		bad[6] += (small != want * 0x01010101u) + (x2 != want * 0x01010101u);
	}
	for (int t = 0; t < 7; ++t)
		if (bad[t])
			atomicAdd(counts + t, bad[t]);
}

} // namespace
} // namespace v7g

using namespace v7g;

extern "C" int v7g_selftest_arith(unsigned long long *dev_counts, void *stream)
{
	if (!dev_counts)
		return set_error(V7G_ERR_ARG, "v7g_selftest_arith: NULL counts");
	DeviceInfo dev;
	int rc = current_device(&dev);
	if (rc != V7G_OK)
		return rc;
	const int grid = resident_grid((const void *)k_selftest, kBlock, 0, 1 << 20, dev);
	const cudaError_t launched = launch_kernel(k_selftest, grid, kBlock, 0, stream, dev_counts);
	return check_launch("v7g_selftest_arith", launched);
}
