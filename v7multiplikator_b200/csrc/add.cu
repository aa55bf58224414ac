// add.cu -- x += y (v7s_add_inplace, add_kernel.inc:26-49) and the
// deterministic synthetic-input generator.
#include "internal.h"
#include "launch.cuh"
#include "reduce.cuh"

namespace v7g {
namespace {

constexpr int kBlock = 256;

template <bool VEC>
__global__ void __launch_bounds__(kBlock) k_add_inplace(float *x, const float *y, int64_t count)
{
	kernel_entry();
	using M = F<false>;
	const int64_t tid = (int64_t)blockIdx.x * kBlock + threadIdx.x;
	const int64_t nthreads = (int64_t)gridDim.x * kBlock;
	if (VEC) {
		float4 *x4 = reinterpret_cast<float4 *>(x);
		const float4 *y4 = reinterpret_cast<const float4 *>(y);
		const int64_t n4 = count >> 2;
		for (int64_t i = tid; i < n4; i += nthreads) {
			float4 a = ld_stream4(x4 + i), b = ld_stream4(y4 + i);
			st_stream4(x4 + i, make_float4(M::add(a.x, b.x), M::add(a.y, b.y), M::add(a.z, b.z), M::add(a.w, b.w)));
		}
		const int64_t t = (n4 << 2) + tid;
		if (tid < (count & 3))
			x[t] = M::add(x[t], y[t]);
	} else {
		for (int64_t i = tid; i < count; i += nthreads)
			x[i] = M::add(x[i], y[i]);
	}
}

// SplitMix64 finaliser (Steele, Lea, Flood, "Fast splittable pseudorandom
// number generators", OOPSLA 2014): a bijective 64-bit mixer.
__device__ __forceinline__ uint64_t mix64(uint64_t z)
{
	z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
	z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
	return z ^ (z >> 31);
}

// Box-Muller from correctly rounded IEEE operations only, so that a host
// program doing the same operations in the same order (the oracle's
// orc_fill_normal) reproduces every value bit for bit.  The logarithm and the
// cosine are evaluated here rather than with the math library, whose results
// are not specified to the last bit:
//   ln u:  u = 2^e * m with m in [sqrt(1/2), sqrt(2)); ln m = 2 atanh(s),
//          s = (m - 1) / (m + 1), |s| < 0.172, odd series to s^11
//          (relative error below 1e-9 before rounding);
//   cos(2 pi v): v*4 = q + f, q the quadrant, f in [0, 1); cos and sin of
//          f * pi/2 by their Taylor series to f^14 and f^13 (error below
//          1e-9), the quadrant picking cos, -sin, -cos or sin.
// The series coefficients are the float32 roundings of (-1)^k (pi/2)^2k/(2k)!,
// (-1)^k (pi/2)^(2k+1)/(2k+1)! and 2/(2k+1).
__device__ __forceinline__ float fill_ln(float u)
{
	using M = F<false>;
	uint32_t b = __float_as_uint(u); // u in [2^-24, 1]: normal, positive
	int e = (int)(b >> 23) - 127;
	b = (b & 0x007fffffu) | 0x3f800000u; // m in [1, 2)
	if (b > 0x3FB504F3u) {                 // m > sqrt(2): m / 2, e + 1
		b -= 0x00800000u;
		e += 1;
	}
	const float m = __uint_as_float(b);
	const float s = M::div(M::sub(m, 1.0f), M::add(m, 1.0f));
	const float x = M::mul(s, s);
	float p = M::fma(x, __uint_as_float(0x3E3A2E8Cu), __uint_as_float(0x3E638E39u));
	p = M::fma(x, p, __uint_as_float(0x3E924925u));
	p = M::fma(x, p, __uint_as_float(0x3ECCCCCDu));
	p = M::fma(x, p, __uint_as_float(0x3F2AAAABu));
	p = M::fma(x, p, 2.0f);
	return M::fma((float)e, __uint_as_float(0x3F317218u), M::mul(s, p));
}

__device__ __forceinline__ float fill_cos2pi(float v)
{
	using M = F<false>;
	const float v4 = M::mul(v, 4.0f); // exact
	const int q = (int)v4;             // 0..3
	const float f = M::sub(v4, (float)q);
	const float x = M::mul(f, f);
	float c = M::fma(x, __uint_as_float(0xB1DB7128u), __uint_as_float(0x34FCE9C5u));
	c = M::fma(x, c, __uint_as_float(0xB7D368F9u));
	c = M::fma(x, c, __uint_as_float(0x3A70FA83u));
	c = M::fma(x, c, __uint_as_float(0xBCAAE9E4u));
	c = M::fma(x, c, __uint_as_float(0x3E81E0F8u));
	c = M::fma(x, c, __uint_as_float(0xBF9DE9E6u));
	c = M::fma(x, c, 1.0f);
	float sn = M::fma(x, __uint_as_float(0x33747A1Au), __uint_as_float(0xB67183A8u));
	sn = M::fma(x, sn, __uint_as_float(0x39283C1Au));
	sn = M::fma(x, sn, __uint_as_float(0xBB996966u));
	sn = M::fma(x, sn, __uint_as_float(0x3DA335E3u));
	sn = M::fma(x, sn, __uint_as_float(0xBF255DE7u));
	sn = M::fma(x, sn, __uint_as_float(0x3FC90FDBu));
	sn = M::mul(f, sn);
	return q == 0 ? c : q == 1 ? -sn : q == 2 ? -c : sn;
}

// N(mean, std) from the counter (seed, row, col) by the Box-Muller transform.
__global__ void __launch_bounds__(kBlock) k_fill_normal(float *dst, int64_t rows, int64_t n, int64_t row0, uint64_t seed, float mean, float std)
{
	kernel_entry();
	using M = F<false>;
	const int64_t total = rows * n;
	const int64_t stride = (int64_t)gridDim.x * kBlock;
	const uint64_t key = mix64(seed ^ 0x9e3779b97f4a7c15ull);
	for (int64_t i = (int64_t)blockIdx.x * kBlock + threadIdx.x; i < total; i += stride) {
		const int64_t r = i / n, c = i - r * n;
		const uint64_t h = mix64(key ^ mix64((uint64_t)(row0 + r) * 0xd1b54a32d192ed03ull + (uint64_t)c));
		const float u1 = M::mul((float)(uint32_t)(h >> 40) + 1.0f, 5.96046448e-08f); // (0, 1], exact
		const float u2 = M::mul((float)(uint32_t)(h & 0xffffffu), 5.96046448e-08f);  // [0, 1), exact
		const float z = M::mul(M::sqrt(M::mul(-2.0f, fill_ln(u1))), fill_cos2pi(u2));
		dst[i] = M::add(mean, M::mul(std, z));
	}
}

// `oversubscribe` x the blocks that fit resident at once (at most
// work_blocks): a few waves of CTAs stream measurably faster on B200 than
// exactly one resident wave.
template <typename Kernel, typename... Args>
int launch_persistent(Kernel kernel, const char *what, int64_t work_blocks, int oversubscribe, void *stream, Args... args)
{
	DeviceInfo dev;
	int rc = current_device(&dev);
	if (rc != V7G_OK)
		return rc;
	work_blocks = work_blocks < 1 ? 1 : work_blocks;
	const int resident = resident_grid((const void *)kernel, kBlock, 0, work_blocks, dev);
	const int grid = (int)(work_blocks < (int64_t)resident * oversubscribe ? work_blocks : (int64_t)resident * oversubscribe);
	const cudaError_t launched = launch_kernel(kernel, grid, kBlock, 0, stream, args...);
	return check_launch(what, launched);
}

} // namespace
} // namespace v7g

using namespace v7g;

extern "C" {

int v7g_add_inplace(float *x, const float *y, int64_t count, void *stream)
{
	if (count < 0)
		return set_error(V7G_ERR_ARG, "v7g_add_inplace: count = %lld < 0", (long long)count);
	if (count == 0)
		return clear_error();
	if (!x || !y)
		return set_error(V7G_ERR_ARG, "v7g_add_inplace: NULL pointer");
	if (aligned16(x) && aligned16(y))
		// a one-shot grid (up to 64 resident waves), as for the elementwise SwiGLU
		return launch_persistent(k_add_inplace<true>, "v7g_add_inplace", ((count >> 2) + kBlock - 1) / kBlock, 64, stream, x, y, count);
	return launch_persistent(k_add_inplace<false>, "v7g_add_inplace", (count + kBlock - 1) / kBlock, 1, stream, x, y, count);
}

int v7g_fill_normal(float *dst, int64_t rows, int64_t n, int64_t row0, uint64_t seed, float mean, float std, void *stream)
{
	if (rows < 0 || n < 0 || row0 < 0)
		return set_error(V7G_ERR_ARG, "v7g_fill_normal: negative rows, n or row0");
	if (rows == 0 || n == 0)
		return clear_error();
	if (!dst)
		return set_error(V7G_ERR_ARG, "v7g_fill_normal: NULL pointer");
	return launch_persistent(k_fill_normal, "v7g_fill_normal", (rows * n + kBlock - 1) / kBlock, 1, stream, dst, rows, n, row0, seed, mean, std);
}

} // extern "C"
