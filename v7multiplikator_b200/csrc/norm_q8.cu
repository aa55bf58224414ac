// norm_q8.cu -- fused RMSNorm -> Q8 over rows of device memory
// (v7s_rmsnorm_quantize, rmsnorm_quantize_kernel.inc:60-218).  An FTZ
// compilation unit: the reference runs the Q8 path with FTZ+DAZ.
#include "internal.h"
#include "launch.cuh"
#include "q8_fast.cuh"
#include "reduce.cuh"

namespace v7g {
namespace {

constexpr int kBlock = 256;
constexpr int kWarpsPerBlock = kBlock / 32;
// four CTAs per SM (at most 64 registers a thread): more rows in flight
constexpr int kMinBlocks = 4;

// The MAXPS tree of one 64-element group (quantize_kernel.inc:62-81) when a
// group sits on 8 consecutive lanes, lane q holding elements 8q..8q+7: the
// reference first reduces the 8-float blocks column by column as
// max(max(max(b0, b1), max(b2, b3)), max(max(b4, b5), max(b6, b7))) -- lanes
// q ^ 1, q ^ 2, q ^ 4 here, the lower block always the first operand -- then
// the 8 columns in-lane: max(c_j, c_{j+4}), then (0, 2), (1, 3), then the
// pair.  x86_max returns its second operand when either is NaN, so the order
// decides which NaN-carrying value survives.
__device__ __forceinline__ float group_absmax8_tree(const float (&a)[8], int q)
{
	float m[8];
#pragma unroll
	for (int c = 0; c < 8; ++c)
		m[c] = a[c];
#pragma unroll
	for (int bit = 1; bit < 8; bit <<= 1) {
#pragma unroll
		for (int c = 0; c < 8; ++c) {
			const float o = __shfl_xor_sync(kFullMask, m[c], bit);
			const bool upper = (q & bit) != 0;
			m[c] = x86_max(upper ? o : m[c], upper ? m[c] : o);
		}
	}
	const float v0 = x86_max(m[0], m[4]), v1 = x86_max(m[1], m[5]), v2 = x86_max(m[2], m[6]), v3 = x86_max(m[3], m[7]);
	return x86_max(x86_max(v0, v2), x86_max(v1, v3));
}

// Group absmax on 8 lanes: without NaN the tree's result is the largest
// magnitude, an integer maximum of the bit patterns; a NaN anywhere in the
// warp sends the warp through the exact tree.  maxbits: the group's largest
// magnitude bit pattern (above 0x7f7fffff when it holds an inf or a NaN).
__device__ __forceinline__ float group_absmax8(const float (&h)[8], int q, uint32_t &maxbits)
{
	float a[8];
	uint32_t mb = 0;
#pragma unroll
	for (int c = 0; c < 8; ++c) {
		a[c] = __uint_as_float(abs_bits(h[c]));
		mb = max(mb, abs_bits(h[c]));
	}
	mb = max(mb, __shfl_xor_sync(kFullMask, mb, 1));
	mb = max(mb, __shfl_xor_sync(kFullMask, mb, 2));
	mb = max(mb, __shfl_xor_sync(kFullMask, mb, 4));
	maxbits = mb;
	if (__any_sync(kFullMask, mb > 0x7f800000u))
		return group_absmax8_tree(a, q);
	return __uint_as_float(mb);
}

// Codes of a group holding an inf or a NaN: the general conversion with its
// range tests.  Out of line so that the common finite case stays a short
// straight path instead of both forms being computed and selected.
__device__ __noinline__ uint2 codes8_general(float4 h0, float4 h1, float recip)
{
	return make_uint2(q8_codes4_x2(h0, recip), q8_codes4_x2(h1, recip));
}

// Pass 1 accumulates the sum of squares in the chain layout (lane l: elements
// l + 32k) in unguarded chunks of C loads.  Pass 2 re-reads the row from L2 in
// the quantiser's layout -- four 64-element groups per warp, eight
// consecutive floats per lane, so the per-group work (absmax reduction,
// scale, reciprocal) is shared by four groups per instruction -- normalises
// as (scale * x) * w and quantises.  Latency is covered by the four resident
// CTAs per SM rather than by prefetch buffers, which cost register moves on
// every element.  x and w must be 16-byte aligned, codes 8-byte aligned.
template <int C>
__global__ void __launch_bounds__(kBlock, kMinBlocks) k_rmsnorm_quantize_rows(uint2 *codes, float *scales, const float *x, const float *__restrict__ w, int64_t rows, int n, float eps)
{
	kernel_entry();
	using M = F<true>;
	const int lane = threadIdx.x & 31;
	const int slot = lane >> 3; // group of the four the warp holds
	const int q = lane & 7;     // eight elements 8q..8q+7 of it
	const int64_t nwarps = ((int64_t)gridDim.x * kBlock) >> 5;
	const int vpl = n >> 5;
	const int ngr = n >> 6;
	const float nf = (float)n;
	const float4 *w4 = reinterpret_cast<const float4 *>(w);
	for (int64_t row = ((int64_t)blockIdx.x * kBlock + threadIdx.x) >> 5; row < rows; row += nwarps) {
		const float *xr = x + row * n + lane;
		float acc = 0.0f;
		// full chunks: C loads in flight per lane, no per-slot guards (the
		// resident warps, not a prefetch buffer, cover the latency)
		int k0 = 0;
		for (; k0 + C <= vpl; k0 += C) {
			float v[C];
#pragma unroll
			for (int k = 0; k < C; ++k)
				v[k] = xr[32 * (k0 + k)];
#pragma unroll
			for (int k = 0; k < C; ++k)
				acc = M::fma(v[k], v[k], acc);
		}
		for (; k0 < vpl; ++k0) {
			const float v = xr[32 * k0];
			acc = M::fma(v, v, acc);
		}
		const float scale = rms_scale<true>(reduce_chains_4x8<true>(acc), nf, eps);
		const float4 *x4 = reinterpret_cast<const float4 *>(x + row * n);
		uint2 *qr = codes + row * (n >> 3);
		float *sr = scales + row * ngr;
		const float2 s2 = splat2(scale);
		auto load = [&](int j, float4 (&xv)[2], float4 (&wv)[2]) {
			const int g = 4 * j + slot;
#pragma unroll
			for (int u = 0; u < 2; ++u) {
				xv[u] = wv[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
				if (g < ngr) {
					xv[u] = ld_stream4(x4 + g * 16 + 2 * q + u);
					wv[u] = __ldg(w4 + g * 16 + 2 * q + u);
				}
			}
		};
		// two rounds of four groups per L2 round trip
		for (int j = 0; 4 * j < ngr; j += 2) {
			float4 xv[2][2], wv[2][2];
			load(j, xv[0], wv[0]);
			load(j + 1, xv[1], wv[1]);
#pragma unroll
			for (int t = 0; t < 2; ++t) {
				if (4 * (j + t) >= ngr) // warp-uniform
					break;
				const int g = 4 * (j + t) + slot;
				// (scale * x) * w, the reference's order (rmsnorm_quantize_kernel.inc:52-57)
				float h[8];
#pragma unroll
				for (int u = 0; u < 2; ++u) {
					const float2 h01 = mul2(mul2(s2, make_float2(xv[t][u].x, xv[t][u].y)), make_float2(wv[t][u].x, wv[t][u].y));
					const float2 h23 = mul2(mul2(s2, make_float2(xv[t][u].z, xv[t][u].w)), make_float2(wv[t][u].z, wv[t][u].w));
					h[4 * u] = h01.x;
					h[4 * u + 1] = h01.y;
					h[4 * u + 2] = h23.x;
					h[4 * u + 3] = h23.y;
				}
				float gscale, recip;
				uint32_t maxbits;
				q8_scale_fast(group_absmax8(h, q, maxbits), gscale, recip);
				if (g < ngr) {
					const float4 h0 = make_float4(h[0], h[1], h[2], h[3]), h1 = make_float4(h[4], h[5], h[6], h[7]);
					// a finite group's products stay within 127.5: the short code path
					uint2 c = make_uint2(q8_codes4_small(h0, recip), q8_codes4_small(h1, recip));
					if (maxbits > 0x7f7fffffu)
						c = codes8_general(h0, h1, recip);
					__stcs(qr + g * 8 + q, c);
					if (q == 0)
						__stcs(sr + g, gscale);
				}
			}
		}
	}
}

// slots per lane per pipelined chunk of the sum-of-squares pass
constexpr int kChunk = 32;

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
	const cudaError_t launched = launch_kernel(kernel, grid, kBlock, 0, stream, args...);
	return check_launch(what, launched);
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
	if ((reinterpret_cast<uintptr_t>(codes) & 7) != 0 || !aligned16(x) || !aligned16(w))
		return set_error(V7G_ERR_ARG, "v7g_rmsnorm_quantize_rows: x and w must be 16-byte aligned, codes 8-byte aligned");
	return launch_rows(k_rmsnorm_quantize_rows<kChunk>, "v7g_rmsnorm_quantize_rows", rows, stream,
	                   reinterpret_cast<uint2 *>(codes), scales, x, w, rows, n, eps);
}

} // extern "C"
