// norm_q8.cu -- fused RMSNorm -> Q8 over rows of device memory
// (v7s_rmsnorm_quantize, rmsnorm_quantize_kernel.inc:60-218).  An FTZ
// compilation unit: the reference runs the Q8 path with FTZ+DAZ.
#include "internal.h"
#include "launch.cuh"
#include "q8_fast.cuh"
#include "reduce.cuh"
#include "rowpipe.cuh"

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

// Rows whose normalised values are all finite take a shorter path.  When the
// row's sum of squares ss and its scale are finite, every |scale * x| is at
// most sqrt(n) (x^2 <= ss; a few ulps of rounding aside), below 4097 for rows
// shorter than 2^24; with every |w| below kTameGamma the products (scale * x)
// * w are then finite too.  For such a group the MAXPS tree's result is the
// plain maximum of the magnitudes, the scale needs no IEEE special case and
// every code comes from the short path.  Whether gamma is tame is decided
// once per CTA.
constexpr float kTameGamma = 1e30f;

__device__ __forceinline__ bool row_is_tame(bool gamma_tame, float ss, float scale)
{
	return gamma_tame && ss <= 3.402823466e38f && scale <= 3.402823466e38f; // false for inf and NaN
}

// Largest magnitude of a group of finite values held eight per lane by eight
// consecutive lanes.
__device__ __forceinline__ float group_absmax8_finite(const float (&h)[8])
{
	float m = fmaxf(fmaxf(fmaxf(fabsf(h[0]), fabsf(h[1])), fmaxf(fabsf(h[2]), fabsf(h[3]))),
	                fmaxf(fmaxf(fabsf(h[4]), fabsf(h[5])), fmaxf(fabsf(h[6]), fabsf(h[7]))));
	m = fmaxf(m, __shfl_xor_sync(kFullMask, m, 1));
	m = fmaxf(m, __shfl_xor_sync(kFullMask, m, 2));
	return fmaxf(m, __shfl_xor_sync(kFullMask, m, 4));
}

__device__ __forceinline__ void norm_h8(float (&h)[8], float4 x0, float4 x1, float4 w0, float4 w1, float2 s2)
{
	const float2 a = mul2(mul2(s2, make_float2(x0.x, x0.y)), make_float2(w0.x, w0.y));
	const float2 b = mul2(mul2(s2, make_float2(x0.z, x0.w)), make_float2(w0.z, w0.w));
	const float2 c = mul2(mul2(s2, make_float2(x1.x, x1.y)), make_float2(w1.x, w1.y));
	const float2 d = mul2(mul2(s2, make_float2(x1.z, x1.w)), make_float2(w1.z, w1.w));
	h[0] = a.x;
	h[1] = a.y;
	h[2] = b.x;
	h[3] = b.y;
	h[4] = c.x;
	h[5] = c.y;
	h[6] = d.x;
	h[7] = d.y;
}

// Whether every |w[i]| of gamma is below kTameGamma (NaN is not), over the
// whole CTA; every thread of the CTA must call it.
__device__ __forceinline__ bool gamma_tame_cta(const float *w, int n)
{
	bool ok = true;
	for (int i = threadIdx.x; i < n; i += blockDim.x)
		ok = ok && fabsf(w[i]) < kTameGamma;
	return __syncthreads_and(ok) != 0;
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
	const bool gtame = gamma_tame_cta(w, n);
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
		const float ss = reduce_chains_4x8<true>(acc);
		const float scale = rms_scale<true>(ss, nf, eps);
		const float4 *x4 = reinterpret_cast<const float4 *>(x + row * n);
		uint2 *qr = codes + row * (n >> 3);
		float *sr = scales + row * ngr;
		const float2 s2 = splat2(scale);
		if (row_is_tame(gtame, ss, scale)) { // warp-uniform
			// two rounds of four groups at a time; their scales in pair arithmetic
			for (int j = 0; 4 * j < ngr; j += 2) {
				float h[2][8];
				bool live[2];
#pragma unroll
				for (int t = 0; t < 2; ++t) {
					const int g = 4 * (j + t) + slot;
					live[t] = g < ngr;
					const int gi = live[t] ? g : 0; // past the row's last group: group 0, nothing stored
					float4 xv[2], wv[2];
#pragma unroll
					for (int u = 0; u < 2; ++u) {
						xv[u] = ld_stream4(x4 + gi * 16 + 2 * q + u);
						wv[u] = __ldg(w4 + gi * 16 + 2 * q + u);
					}
					norm_h8(h[t], xv[0], xv[1], wv[0], wv[1], s2);
				}
				float2 gscale, recip;
				q8_scale_finite2(group_absmax8_finite(h[0]), group_absmax8_finite(h[1]), gscale, recip);
#pragma unroll
				for (int t = 0; t < 2; ++t) {
					if (!live[t])
						continue;
					const int g = 4 * (j + t) + slot;
					const float r = t ? recip.y : recip.x;
					__stcs(qr + g * 8 + q, make_uint2(q8_codes4_small(make_float4(h[t][0], h[t][1], h[t][2], h[t][3]), r),
					                                  q8_codes4_small(make_float4(h[t][4], h[t][5], h[t][6], h[t][7]), r)));
					if (q == 0)
						__stcs(sr + g, t ? gscale.y : gscale.x);
				}
			}
			continue;
		}
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

// The same on the row pipeline (rowpipe.cuh): the row is in shared memory, so
// pass 2 reads it in an order free of bank conflicts -- lane q of a group's
// eight takes elements 4q..4q+3 and 32+4q..32+4q+3 -- and the rare group
// that needs the exact MAXPS tree (a NaN in the warp) re-reads its elements
// in the reference's block order (lane q: 8q..8q+7) for the tree alone.  Same
// arithmetic in the same order as k_rmsnorm_quantize_rows.  Codes and scales
// are written with ordinary stores (a row's codes are a quarter of its
// bytes).  x, w 16-byte aligned; codes 4-byte aligned.
// One slot per warp, so that sixteen warps fit beside the slots: the
// quantiser pass is latency-bound, and more warps hide more of it than more
// rows in flight per warp do.  Measured on B200 at n = 2048, back to back,
// inputs larger than L2 (2048 / 4096 / 16384 rows): one slot and 16 warps 6.95
// / 11.3 / 32.5 us, three slots and 8 warps 8.6 / 13.0 / 32.4 us, two slots and
// 13 warps 8.5 / 13.9 / 32.4 us, one slot and 20 warps 7.3 / 12.0 / 32.1 us.
constexpr int kRmsqPipeStages = 1;

template <int S>
__global__ void __launch_bounds__(kPipeMaxWarps * 32, 1) k_rmsnorm_quantize_pipe(uint32_t *codes, float *scales, const float *x, const float *w, int64_t rows, int n, float eps)
{
	extern __shared__ __align__(128) unsigned char smem[];
	using M = F<true>;
	const int W = blockDim.x >> 5;
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int gs = lane >> 3; // group of the four the warp holds
	const int q = lane & 7;
	const PipeLayout L = pipe_layout(n, 1, W, S);
	const int64_t nw = (int64_t)gridDim.x * W;
	// rows interleaved over the CTAs first: CTA b holds rows b, b + G, b + 2G,
	// ... (every SM within one row of the average), its warp w the ones from
	// b + G w on, every G W
	const int64_t first = (int64_t)warp * gridDim.x + blockIdx.x;
	const float *const src[1] = {x};
	WarpPipe<S, 1> p = pipe_start<S, 1>(smem, L, src, w, n, first, nw, rows);
	const float4 *w4 = reinterpret_cast<const float4 *>(smem);
	bool ok = pipe_wait_gamma(p, smem, L, first, nw, rows);
	const bool gtame = gamma_tame_cta(reinterpret_cast<const float *>(smem), n);
	const int vpl = n >> 5, ngr = n >> 6;
	const float nf = (float)n;
	for (int64_t row = first; ok && row < rows; row += nw) {
		const float *xs = p.slot((int)(p.waited % S), 0);
		if (!p.wait()) {
			ok = false;
			break;
		}
		float acc = 0.0f;
#pragma unroll 8
		for (int k = 0; k < vpl; ++k) {
			const float v = xs[lane + 32 * k];
			acc = M::fma(v, v, acc);
		}
		const float ss = reduce_chains_4x8<true>(acc);
		const float scale = rms_scale<true>(ss, nf, eps);
		const float2 s2 = splat2(scale);
		const float4 *x4 = reinterpret_cast<const float4 *>(xs);
		uint32_t *qr = codes + row * (n >> 2);
		float *sr = scales + row * ngr;
		if (row_is_tame(gtame, ss, scale)) { // warp-uniform
			for (int j = 0; 4 * j < ngr; j += 2) {
				float h[2][8];
				bool live[2];
#pragma unroll
				for (int t = 0; t < 2; ++t) {
					const int g = 4 * (j + t) + gs;
					live[t] = g < ngr;
					const int gi = live[t] ? g : 0;
					norm_h8(h[t], x4[gi * 16 + q], x4[gi * 16 + 8 + q], w4[gi * 16 + q], w4[gi * 16 + 8 + q], s2);
				}
				float2 gscale, recip;
				q8_scale_finite2(group_absmax8_finite(h[0]), group_absmax8_finite(h[1]), gscale, recip);
#pragma unroll
				for (int t = 0; t < 2; ++t) {
					if (!live[t])
						continue;
					const int g = 4 * (j + t) + gs;
					const float r = t ? recip.y : recip.x;
					__stcs(qr + g * 16 + q, q8_codes4_small(make_float4(h[t][0], h[t][1], h[t][2], h[t][3]), r));
					__stcs(qr + g * 16 + 8 + q, q8_codes4_small(make_float4(h[t][4], h[t][5], h[t][6], h[t][7]), r));
					if (q == 0)
						__stcs(sr + g, t ? gscale.y : gscale.x);
				}
			}
			__syncwarp(); // every lane is done with the slot before it is refilled
			const int64_t next = row + S * nw;
			if (next < rows)
				p.issue(next, lane == 0);
			continue;
		}
#pragma unroll 2
		for (int j = 0; 4 * j < ngr; ++j) { // warp-uniform
			const int g = 4 * j + gs;
			const bool live = g < ngr;
			const int gi = live ? g : 0; // a lane past the row's last group reads group 0, stores nothing
			float h[8];
			norm_h8(h, x4[gi * 16 + q], x4[gi * 16 + 8 + q], w4[gi * 16 + q], w4[gi * 16 + 8 + q], s2);
			uint32_t mb = 0;
#pragma unroll
			for (int c = 0; c < 8; ++c)
				mb = max(mb, abs_bits(h[c]));
			mb = max(mb, __shfl_xor_sync(kFullMask, mb, 1));
			mb = max(mb, __shfl_xor_sync(kFullMask, mb, 2));
			mb = max(mb, __shfl_xor_sync(kFullMask, mb, 4));
			float wmax = __uint_as_float(mb);
			if (__any_sync(kFullMask, mb > 0x7f800000u)) {
				// the exact tree wants lane q to hold the 8-float block q
				float hb[8], a[8];
				norm_h8(hb, x4[gi * 16 + 2 * q], x4[gi * 16 + 2 * q + 1], w4[gi * 16 + 2 * q], w4[gi * 16 + 2 * q + 1], s2);
#pragma unroll
				for (int c = 0; c < 8; ++c)
					a[c] = __uint_as_float(abs_bits(hb[c]));
				wmax = group_absmax8_tree(a, q);
			}
			float gscale, recip;
			q8_scale_fast(wmax, gscale, recip);
			if (live) {
				const float4 h0 = make_float4(h[0], h[1], h[2], h[3]), h1 = make_float4(h[4], h[5], h[6], h[7]);
				uint2 c = make_uint2(q8_codes4_small(h0, recip), q8_codes4_small(h1, recip));
				if (mb > 0x7f7fffffu)
					c = codes8_general(h0, h1, recip);
				__stcs(qr + g * 16 + q, c.x);
				__stcs(qr + g * 16 + 8 + q, c.y);
				if (q == 0)
					__stcs(sr + g, gscale);
			}
		}
		__syncwarp(); // every lane is done with the slot before it is refilled
		const int64_t next = row + S * nw;
		if (next < rows)
			p.issue(next, lane == 0);
	}
	if (!ok)
		p.drain();
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

uint64_t g_smem_rmsq = 0;

template <int S>
int launch_rmsq_pipe(int8_t *codes, float *scales, const float *x, const float *w, int64_t rows, int n, float eps, void *stream)
{
	DeviceInfo dev;
	int rc = current_device(&dev);
	if (rc != V7G_OK)
		return rc;
	const int W = pipe_warps_for(n, 1, S, rows, dev.sm_count);
	if (W == 0 || pipe_allow_smem(k_rmsnorm_quantize_pipe<S>, dev.device, g_smem_rmsq) != 0)
		return V7G_ERR_UNSUPPORTED;
	const int64_t want = (rows + W - 1) / W;
	const int grid = (int)(want < dev.sm_count ? want : dev.sm_count);
	const cudaError_t launched = launch_kernel(k_rmsnorm_quantize_pipe<S>, grid, W * 32, pipe_layout(n, 1, W, S).total(), stream,
	                                           reinterpret_cast<uint32_t *>(codes), scales, x, w, rows, n, eps);
	return check_launch("v7g_rmsnorm_quantize_rows", launched);
}

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
	if (rows > 256 && aligned16(codes)) {
		const int rc = launch_rmsq_pipe<kRmsqPipeStages>(codes, scales, x, w, rows, n, eps, stream);
		if (rc != V7G_ERR_UNSUPPORTED)
			return rc;
	}
	return launch_rows(k_rmsnorm_quantize_rows<kChunk>, "v7g_rmsnorm_quantize_rows", rows, stream,
	                   reinterpret_cast<uint2 *>(codes), scales, x, w, rows, n, eps);
}

} // extern "C"

namespace v7g {
// Given-up waits of this unit's row pipeline (added into v7g_pipeline_timeouts).
unsigned int norm_q8_pipe_timeouts() { return rowpipe_timeouts_here(); }
} // namespace v7g
