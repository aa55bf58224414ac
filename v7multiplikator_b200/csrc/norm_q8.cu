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

// Pass 1 accumulates the sum of squares in the chain layout (lane l: elements
// l + 32k, pipelined as in norm.cu).  Pass 2 re-reads the row from L2 in the
// quantiser's layout -- each 64-element group on a half-warp, a float4 per
// lane, as in k_q8_groups -- normalises it as (scale * x) * w and quantises,
// loads of the next group pair issued before the current one is processed.
// x, w and codes must be 16-byte aligned.
template <int C>
__global__ void __launch_bounds__(kBlock) k_rmsnorm_quantize_rows(uint32_t *codes, float *scales, const float *x, const float *__restrict__ w, int64_t rows, int n, float eps)
{
	using M = F<true>;
	const int lane = threadIdx.x & 31;
	const int half = lane >> 4;
	const int hl = lane & 15;
	const int64_t nwarps = ((int64_t)gridDim.x * kBlock) >> 5;
	const int vpl = n >> 5;
	const int ngr = n >> 6;
	const float nf = (float)n;
	const float4 *w4 = reinterpret_cast<const float4 *>(w);
	for (int64_t row = ((int64_t)blockIdx.x * kBlock + threadIdx.x) >> 5; row < rows; row += nwarps) {
		const float *xr = x + row * n + lane;
		float acc = 0.0f;
		float v[C];
#pragma unroll
		for (int k = 0; k < C; ++k)
			if (k < vpl)
				v[k] = xr[32 * k];
		for (int k0 = 0; k0 < vpl; k0 += C) {
			float vn[C];
#pragma unroll
			for (int k = 0; k < C; ++k)
				if (k0 + C + k < vpl)
					vn[k] = xr[32 * (k0 + C + k)];
#pragma unroll
			for (int k = 0; k < C; ++k)
				if (k0 + k < vpl)
					acc = M::fma(v[k], v[k], acc);
#pragma unroll
			for (int k = 0; k < C; ++k)
				v[k] = vn[k];
		}
		const float scale = rms_scale<true>(reduce_chains_4x8<true>(acc), nf, eps);
		const float4 *x4 = reinterpret_cast<const float4 *>(x + row * n);
		uint32_t *qr = codes + row * (n >> 2);
		float *sr = scales + row * ngr;
		const float2 s2 = splat2(scale);
		auto load = [&](int j, float4 &xv, float4 &wv) {
			const int g = 2 * j + half;
			xv = wv = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
			if (g < ngr) {
				xv = ld_stream4(x4 + g * 16 + hl);
				wv = __ldg(w4 + g * 16 + hl);
			}
		};
		float4 xv, wv;
		load(0, xv, wv);
		for (int j = 0; 2 * j < ngr; ++j) {
			float4 xn, wn;
			load(j + 1, xn, wn);
			const int g = 2 * j + half;
			// (scale * x) * w, the reference's order (rmsnorm_quantize_kernel.inc:52-57)
			const float2 h01 = mul2(mul2(s2, make_float2(xv.x, xv.y)), make_float2(wv.x, wv.y));
			const float2 h23 = mul2(mul2(s2, make_float2(xv.z, xv.w)), make_float2(wv.z, wv.w));
			const float4 h = make_float4(h01.x, h01.y, h23.x, h23.y);
			float gscale, recip;
			q8_scale_fast(group_absmax_f4(h, lane), gscale, recip);
			if (g < ngr) {
				__stcs(qr + g * 16 + hl, q8_codes4_x2(h, recip));
				if (hl == 0)
					__stcs(sr + g, gscale);
			}
			xv = xn;
			wv = wn;
		}
	}
}

// slots per lane per pipelined chunk of the sum-of-squares pass
constexpr int kChunk = 16;

template <typename Kernel, typename... Args>
int launch_rows(Kernel kernel, const char *what, int64_t rows, void *stream, Args... args)
{
	DeviceInfo dev;
	int rc = current_device(&dev);
	if (rc != V7G_OK)
		return rc;
	const int64_t want = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
	const int resident = resident_grid((const void *)kernel, kBlock, 0, want, dev);
	const int grid = (int)(want < 2ll * resident ? want : 2ll * resident);
	kernel<<<grid, kBlock, 0, (cudaStream_t)stream>>>(args...);
	return check_launch(what);
}

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
	if (!aligned16(codes) || !aligned16(x) || !aligned16(w))
		return set_error(V7G_ERR_ARG, "v7g_rmsnorm_quantize_rows: codes, x and w must be 16-byte aligned");
	return launch_rows(k_rmsnorm_quantize_rows<kChunk>, "v7g_rmsnorm_quantize_rows", rows, stream,
	                   reinterpret_cast<uint32_t *>(codes), scales, x, w, rows, n, eps);
}

} // extern "C"
