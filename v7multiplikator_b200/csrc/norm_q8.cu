// norm_q8.cu -- fused RMSNorm -> Q8 over rows of device memory
// (v7s_rmsnorm_quantize, rmsnorm_quantize_kernel.inc:60-218).  An FTZ
// compilation unit: the reference runs the Q8 path with FTZ+DAZ.
#include "internal.h"
#include "q8_fast.cuh"
#include "reduce.cuh"

namespace v7g {
namespace {

constexpr int kBlock = 256;
constexpr int kWarpsPerBlock = kBlock / 32;

// The sum of squares needs the chain layout (lane l: elements l + 32k); the
// quantiser wants each 64-element group on a half-warp as float4s (as in
// k_q8_groups).  The normalised row goes through the warp's slice of shared
// memory in chunks of kQChunk elements: written in chain order (conflict-free
// scalar stores), read back as float4s (conflict-free), so every activation
// is still read from HBM once.  Codes must be 16-byte aligned (4-byte stores).
constexpr int kQChunk = 2048;

template <int CACHE>
__global__ void __launch_bounds__(kBlock) k_rmsnorm_quantize_rows(uint32_t *codes, float *scales, const float *x, const float *__restrict__ w, int64_t rows, int n, float eps)
{
	using M = F<true>;
	extern __shared__ float4 smem4[];
	const int lane = threadIdx.x & 31;
	const int half = lane >> 4;
	const int hl = lane & 15;
	float *stage = reinterpret_cast<float *>(smem4) + (threadIdx.x >> 5) * kQChunk;
	const float4 *stage4 = reinterpret_cast<const float4 *>(stage);
	const int64_t nwarps = ((int64_t)gridDim.x * kBlock) >> 5;
	const int vpl = n >> 5;
	const float nf = (float)n;
	for (int64_t row = ((int64_t)blockIdx.x * kBlock + threadIdx.x) >> 5; row < rows; row += nwarps) {
		const float *xr = x + row * n + lane;
		float v[CACHE];
#pragma unroll
		for (int k = 0; k < CACHE; ++k)
			if (k < vpl)
				v[k] = ld_stream(xr + 32 * k);
		float acc = 0.0f;
#pragma unroll
		for (int k = 0; k < CACHE; ++k)
			if (k < vpl)
				acc = M::fma(v[k], v[k], acc);
		for (int k = CACHE; k < vpl; ++k) {
			float t = ld_stream(xr + 32 * k);
			acc = M::fma(t, t, acc);
		}
		const float scale = rms_scale<true>(reduce_chains_4x8<true>(acc), nf, eps);
		uint32_t *qr = codes + row * (n >> 2);
		float *sr = scales + row * (n >> 6);
		for (int c0 = 0; c0 < n; c0 += kQChunk) {
			const int len = min(kQChunk, n - c0);
			// normalise: (scale * x) * w, the reference's order
#pragma unroll
			for (int k = 0; k < kQChunk / 32; ++k)
				if (32 * k < len) {
					const int e = c0 + 32 * k;
					float xv;
					if (k < CACHE && c0 == 0)
						xv = v[k < CACHE ? k : 0]; // register copy of the first chunk
					else
						xv = ld_stream(xr + e);
					stage[32 * k + lane] = M::mul(M::mul(scale, xv), __ldg(w + e + lane));
				}
			__syncwarp();
			for (int gp = 0; 128 * gp < len; ++gp) {
				const int gl = 2 * gp + half; // group within the chunk
				const bool valid = 64 * gl < len;
				const float4 h = valid ? stage4[gl * 16 + hl] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
				float gscale, recip;
				q8_scale_fast(group_absmax_f4(h, lane), gscale, recip);
				if (valid) {
					const int g = (c0 >> 6) + gl;
					__stcs(qr + g * 16 + hl, q8_codes4_x2(h, recip));
					if (hl == 0)
						__stcs(sr + g, gscale);
				}
			}
			__syncwarp();
		}
	}
}

// Register budget: the smallest slot count that holds the row, up to 64.
int row_cache_slots(int vpl) { return vpl <= 8 ? 8 : vpl <= 16 ? 16 : vpl <= 32 ? 32 : 64; }

// Same, with `smem` bytes of dynamic shared memory per block.
template <typename Kernel, typename... Args>
int launch_rows_smem(Kernel kernel, const char *what, int64_t rows, int smem, void *stream, Args... args)
{
	DeviceInfo dev;
	int rc = current_device(&dev);
	if (rc != V7G_OK)
		return rc;
	if (cudaFuncSetAttribute((const void *)kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
		return set_error(V7G_ERR_CUDA, "%s: cannot reserve %d bytes of shared memory: %s", what, smem, cudaGetErrorString(cudaGetLastError()));
	const int64_t want = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
	const int grid = resident_grid((const void *)kernel, kBlock, smem, want, dev);
	kernel<<<grid, kBlock, smem, (cudaStream_t)stream>>>(args...);
	return check_launch(what);
}

// the per-warp staging slices of k_rmsnorm_quantize_rows
constexpr int kStageBytes = kWarpsPerBlock * kQChunk * (int)sizeof(float);

bool row_len_ok(int n) { return n > 0 && n < (1 << 24); }

} // namespace
} // namespace v7g

using namespace v7g;

extern "C" {

int v7g_rmsnorm_quantize_rows(int8_t *codes, float *scales, const float *x, const float *w, int64_t rows, int n, float eps, void *stream)
{
	if (!row_len_ok(n) || n % 64 != 0)
		return set_error(V7G_ERR_ARG, "v7g_rmsnorm_quantize_rows: n = %d must be a positive multiple of 64 below 2^24", n);
	if (rows < 0)
		return set_error(V7G_ERR_ARG, "v7g_rmsnorm_quantize_rows: rows = %lld < 0", (long long)rows);
	if (rows == 0)
		return clear_error();
	if (!codes || !scales || !x || !w)
		return set_error(V7G_ERR_ARG, "v7g_rmsnorm_quantize_rows: NULL pointer");
	if (!aligned16(codes))
		return set_error(V7G_ERR_ARG, "v7g_rmsnorm_quantize_rows: codes must be 16-byte aligned");
	uint32_t *c4 = reinterpret_cast<uint32_t *>(codes);
	const char *what = "v7g_rmsnorm_quantize_rows";
	switch (row_cache_slots(n / 32)) {
	case 8:
		return launch_rows_smem(k_rmsnorm_quantize_rows<8>, what, rows, kStageBytes, stream, c4, scales, x, w, rows, n, eps);
	case 16:
		return launch_rows_smem(k_rmsnorm_quantize_rows<16>, what, rows, kStageBytes, stream, c4, scales, x, w, rows, n, eps);
	case 32:
		return launch_rows_smem(k_rmsnorm_quantize_rows<32>, what, rows, kStageBytes, stream, c4, scales, x, w, rows, n, eps);
	default:
		return launch_rows_smem(k_rmsnorm_quantize_rows<64>, what, rows, kStageBytes, stream, c4, scales, x, w, rows, n, eps);
	}
}

} // extern "C"
