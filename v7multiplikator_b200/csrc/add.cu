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

// N(mean, std) from the counter (seed, row, col) by the Box-Muller transform.
__global__ void __launch_bounds__(kBlock) k_fill_normal(float *dst, int64_t rows, int64_t n, int64_t row0, uint64_t seed, float mean, float std)
{
	kernel_entry();
	const int64_t total = rows * n;
	const int64_t stride = (int64_t)gridDim.x * kBlock;
	const uint64_t key = mix64(seed ^ 0x9e3779b97f4a7c15ull);
	for (int64_t i = (int64_t)blockIdx.x * kBlock + threadIdx.x; i < total; i += stride) {
		const int64_t r = i / n, c = i - r * n;
		const uint64_t h = mix64(key ^ mix64((uint64_t)(row0 + r) * 0xd1b54a32d192ed03ull + (uint64_t)c));
		const float u1 = ((float)(uint32_t)(h >> 40) + 1.0f) * (1.0f / 16777216.0f); // (0, 1]
		const float u2 = (float)(uint32_t)(h & 0xffffffu) * (1.0f / 16777216.0f);     // [0, 1)
		const float z = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
		dst[i] = mean + std * z;
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
