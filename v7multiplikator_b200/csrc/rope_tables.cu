// rope_tables.cu -- the RoPE cos/sin tables on the device.
//
// The reference fills its tables once at start-up on the x87 unit
// (fused_f32_kernel.inc:257-302): for position p and pair j the angle
// freq_j * p is formed at extended precision (64-bit significand), fsincos
// evaluates it, and both results are stored as fp32.  The frequencies freq_j
// (doubles) come from the host (v7g_rope_freqs, the same x87 sequence as the
// reference).  Here one thread computes one table entry:
//
//   1. the angle at extended precision, exactly as the x87 multiply rounds it:
//      the double product hi = RN53(f * p) and its exact remainder
//      e = fma(f, p, -hi) give f * p = hi + e; rounding that to 64 significant
//      bits keeps e to a multiple of q = ulp(hi) / 2^11 (q / 2 when hi is a
//      power of two and e < 0, the binade below), ties to even;
//   2. sin and cos of hi in double precision (CUDA's sincos, within 2 ulp),
//      then the first-order correction for the low part lo:
//      sin(hi + lo) = sin(hi) + cos(hi) * lo, cos(hi + lo) = cos(hi) - sin(hi) * lo
//      (|lo| < 2^-36 here, so the next term is below 2^-73);
//   3. one rounding to fp32.
//
// The result is the correctly rounded fp32 of the extended-precision angle's
// sine / cosine except when that value lies within about 2^-50 (relative) of a
// rounding boundary; fsincos has its own last-bit error, so the two can differ
// by one fp32 ulp on such entries (one entry in 16.8 million for the
// 131072 x 64 table with base 1e6).
#include "internal.h"
#include "launch.cuh"

namespace v7g {
namespace {

constexpr int kBlock = 256;
constexpr int kMaxHalf = 256;

struct Freqs {
	double f[kMaxHalf];
};

__global__ void __launch_bounds__(kBlock) k_rope_tables(float *cos_t, float *sin_t, int64_t pos0, int64_t positions, int half, int stride, Freqs fr)
{
	kernel_entry();
	const int64_t total = positions * stride;
	const int64_t step = (int64_t)gridDim.x * kBlock;
	for (int64_t i = (int64_t)blockIdx.x * kBlock + threadIdx.x; i < total; i += step) {
		const int64_t r = i / stride;
		const int j = (int)(i - r * stride);
		if (j >= half) {
			cos_t[i] = 0.0f;
			sin_t[i] = 0.0f;
			continue;
		}
		const double f = fr.f[j];
		const double p = (double)(pos0 + r);
		const double hi = __dmul_rn(f, p);
		const double e = __fma_rn(f, p, -hi);
		double lo = 0.0;
		const long long bits = __double_as_longlong(hi) & 0x7fffffffffffffffll;
		const int ex = (int)(bits >> 52);
		if (e != 0.0 && ex > 64 && ex < 2047) {
			// q = 2^(ex - 1023 - 63): 64-bit significand quantum of hi's binade
			double q = __longlong_as_double((long long)(ex - 63) << 52);
			double inv_q = __longlong_as_double((long long)(2109 - ex) << 52);
			if ((bits & 0x000fffffffffffffll) == 0 && e < 0.0) {
				q *= 0.5;
				inv_q *= 2.0;
			}
			lo = rint(e * inv_q) * q;
		}
		double s, c;
		sincos(hi, &s, &c);
		cos_t[i] = __double2float_rn(__fma_rn(-s, lo, c));
		sin_t[i] = __double2float_rn(__fma_rn(c, lo, s));
	}
}

} // namespace
} // namespace v7g

using namespace v7g;

extern "C" int v7g_rope_tables(float *cos_table, float *sin_table, int64_t pos0, int64_t positions, int half, int stride, const double *freqs, void *stream)
{
	const char *what = "v7g_rope_tables";
	if (half <= 0 || half > kMaxHalf || stride < half || positions < 0 || pos0 < 0 || pos0 + positions > ((int64_t)1 << 31))
		return set_error(V7G_ERR_ARG, "%s: need 0 < half <= %d, stride >= half, 0 <= pos0, pos0 + positions <= 2^31", what, kMaxHalf);
	if (!freqs)
		return set_error(V7G_ERR_ARG, "%s: NULL frequencies", what);
	if (positions == 0)
		return clear_error();
	if (!cos_table || !sin_table)
		return set_error(V7G_ERR_ARG, "%s: NULL table", what);
	DeviceInfo dev;
	int rc = current_device(&dev);
	if (rc != V7G_OK)
		return rc;
	Freqs fr;
	for (int j = 0; j < kMaxHalf; ++j)
		fr.f[j] = j < half ? freqs[j] : 0.0;
	const int64_t work_blocks = (positions * stride + kBlock - 1) / kBlock;
	const int resident = resident_grid((const void *)k_rope_tables, kBlock, 0, work_blocks, dev);
	const int grid = (int)(work_blocks < 4ll * resident ? work_blocks : 4ll * resident);
	const cudaError_t launched = launch_kernel(k_rope_tables, grid, kBlock, 0, stream, cos_table, sin_table, pos0, positions, half, stride, fr);
	return check_launch(what, launched);
}
