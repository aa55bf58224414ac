// norm.cu -- RMSNorm and fused residual-add + RMSNorm over rows of device
// memory, one warp per row.
//
// Lane l owns sum-of-squares chain l of the reference's 4 x 8 FMA accumulator
// layout (element e belongs to chain e % 32) and reads its elements e = l + 32k
// with coalesced 128-byte warp accesses.  HBM-bound: algorithmic bytes per row
// = 4n read + 4n written (+ 4n each for the residual of the fused add); the
// second pass's re-read of the row is served by L2, gamma by L1/L2.
#include "internal.h"
#include "launch.cuh"
#include "reduce.cuh"
#include "rowpipe.cuh"

namespace v7g {
namespace {

constexpr int kBlock = 256;
// four CTAs per SM (at most 64 registers a thread): 4096 rows of one warp each
// fit in one wave on 148 SMs, with no half-empty second wave
constexpr int kMinBlocks = 4;

// --- A1  RMSNorm rows (rmsnorm_kernel.inc:12-75), caller's MXCSR: no FTZ ---
// Two passes over the row in chunks of C slots per lane: pass 1 accumulates
// the chains, pass 2 re-reads the row (from L2) to write the output.  A chunk
// issues its C loads before any arithmetic; full chunks carry no per-slot
// guards, and the latency between chunks is covered by the four resident CTAs
// per SM (a register prefetch buffer costs a move per element and registers
// that would lower residency).
template <int C, int MINB = kMinBlocks, int BLOCK = kBlock>
__global__ void __launch_bounds__(BLOCK, MINB) k_rmsnorm_rows(float *o, const float *x, const float *__restrict__ w, int64_t rows, int n, float eps)
{
	kernel_entry();
	using M = F<false>;
	const int lane = threadIdx.x & 31;
	const int64_t nwarps = ((int64_t)gridDim.x * BLOCK) >> 5;
	const int vpl = n >> 5;
	const float nf = (float)n;
	for (int64_t row = ((int64_t)blockIdx.x * BLOCK + threadIdx.x) >> 5; row < rows; row += nwarps) {
		const float *xr = x + row * n + lane;
		float *orow = o + row * n + lane;
		float acc = 0.0f;
		if (vpl == C) {
			// the whole row is one chunk: keep it in registers for the output
			float v[C];
#pragma unroll
			for (int k = 0; k < C; ++k)
				v[k] = ld_stream(xr + 32 * k);
#pragma unroll
			for (int k = 0; k < C; ++k)
				acc = M::fma(v[k], v[k], acc);
			const float scale = rms_scale<false>(reduce_chains_4x8<false>(acc), nf, eps);
#pragma unroll
			for (int k = 0; k < C; ++k)
				st_stream(orow + 32 * k, M::mul(M::mul(v[k], scale), __ldg(w + lane + 32 * k)));
			continue;
		}
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
		const float scale = rms_scale<false>(reduce_chains_4x8<false>(acc), nf, eps);
		for (k0 = 0; k0 + C <= vpl; k0 += C) {
			float v[C];
#pragma unroll
			for (int k = 0; k < C; ++k)
				v[k] = ld_stream(xr + 32 * (k0 + k));
#pragma unroll
			for (int k = 0; k < C; ++k)
				st_stream(orow + 32 * (k0 + k), M::mul(M::mul(v[k], scale), __ldg(w + lane + 32 * (k0 + k))));
		}
		for (; k0 < vpl; ++k0)
			st_stream(orow + 32 * k0, M::mul(M::mul(ld_stream(xr + 32 * k0), scale), __ldg(w + lane + 32 * k0)));
	}
}

// --- A2  fused residual-add + RMSNorm rows (add_rmsnorm_kernel.inc:15-129) ---
// When n/8 is not a multiple of 4 the reference first folds the L = (n/8) % 4
// leading blocks into accumulator A (lanes 0..7 here), then runs the 4-way
// groups from block L on; chain lane l then covers e = 8L + l + 32k.  Pass 1
// writes the new residual as it goes; pass 2 re-reads it (L2) for the output;
// both in unguarded chunks as in k_rmsnorm_rows.
// VEC: pass 2 -- elementwise, so free of the chain layout -- reads the new
// residual and gamma and writes the output as float4 (rows 16-byte aligned),
// a quarter of the load/store instructions of 4-byte lanes; the lanes then
// read residual values other lanes wrote in pass 1, hence the __syncwarp.
template <int C, int MINB = kMinBlocks, int BLOCK = kBlock, bool VEC = false>
__global__ void __launch_bounds__(BLOCK, MINB) k_fused_add_rmsnorm_rows(float *o, float *res, const float *add, const float *__restrict__ w, int64_t rows, int n, float eps)
{
	kernel_entry();
	using M = F<false>;
	const int lane = threadIdx.x & 31;
	const int64_t nwarps = ((int64_t)gridDim.x * BLOCK) >> 5;
	const int left = (n >> 3) & 3;
	const int off = 8 * left;
	const int vpl = (n - off) >> 5;
	const float nf = (float)n;
	for (int64_t row = ((int64_t)blockIdx.x * BLOCK + threadIdx.x) >> 5; row < rows; row += nwarps) {
		float *rr = res + row * n;
		const float *ar = add + row * n;
		float *orow = o + row * n;
		float acc = 0.0f;
		if (left != 0 && lane < 8) {
			for (int b = 0; b < left; ++b) {
				const float s = M::add(ld_stream(rr + 8 * b + lane), ld_stream(ar + 8 * b + lane));
				rr[8 * b + lane] = s;
				acc = M::fma(s, s, acc);
			}
		}
		float *rm = rr + off + lane;
		const float *am = ar + off + lane;
		int k0 = 0;
		for (; k0 + C <= vpl; k0 += C) {
			float r[C], a[C];
#pragma unroll
			for (int k = 0; k < C; ++k) {
				r[k] = ld_stream(rm + 32 * (k0 + k));
				a[k] = ld_stream(am + 32 * (k0 + k));
			}
#pragma unroll
			for (int k = 0; k < C; ++k) {
				const float sv = M::add(r[k], a[k]);
				acc = M::fma(sv, sv, acc);
				rm[32 * (k0 + k)] = sv;
			}
		}
		for (; k0 < vpl; ++k0) {
			const float sv = M::add(ld_stream(rm + 32 * k0), ld_stream(am + 32 * k0));
			acc = M::fma(sv, sv, acc);
			rm[32 * k0] = sv;
		}
		const float scale = rms_scale<false>(reduce_chains_4x8<false>(acc), nf, eps);
		if (VEC) {
			__syncwarp(); // the lanes' residual stores are visible to the whole warp
			const float4 *r4 = reinterpret_cast<const float4 *>(rr);
			const float4 *w4 = reinterpret_cast<const float4 *>(w);
			float4 *o4 = reinterpret_cast<float4 *>(orow);
			const int n4 = n >> 2;
			int i = lane;
			for (; i + 32 * (C / 2 - 1) < n4; i += 32 * (C / 2)) {
				float4 v[C / 2];
#pragma unroll
				for (int k = 0; k < C / 2; ++k)
					v[k] = r4[i + 32 * k];
#pragma unroll
				for (int k = 0; k < C / 2; ++k) {
					const float4 g = __ldg(w4 + i + 32 * k);
					st_stream4(o4 + i + 32 * k, make_float4(M::mul(M::mul(v[k].x, scale), g.x), M::mul(M::mul(v[k].y, scale), g.y),
					                                        M::mul(M::mul(v[k].z, scale), g.z), M::mul(M::mul(v[k].w, scale), g.w)));
				}
			}
			for (; i < n4; i += 32) {
				const float4 v = r4[i], g = __ldg(w4 + i);
				st_stream4(o4 + i, make_float4(M::mul(M::mul(v.x, scale), g.x), M::mul(M::mul(v.y, scale), g.y), M::mul(M::mul(v.z, scale), g.z),
				                               M::mul(M::mul(v.w, scale), g.w)));
			}
			continue;
		}
		if (left != 0 && lane < 8) {
			for (int b = 0; b < left; ++b)
				st_stream(orow + 8 * b + lane, M::mul(M::mul(rr[8 * b + lane], scale), __ldg(w + 8 * b + lane)));
		}
		float *om = orow + off + lane;
		const float *wm = w + off + lane;
		for (k0 = 0; k0 + C <= vpl; k0 += C) {
			float v[C];
#pragma unroll
			for (int k = 0; k < C; ++k)
				v[k] = rm[32 * (k0 + k)];
#pragma unroll
			for (int k = 0; k < C; ++k)
				st_stream(om + 32 * (k0 + k), M::mul(M::mul(v[k], scale), __ldg(wm + 32 * (k0 + k))));
		}
		for (; k0 < vpl; ++k0)
			st_stream(om + 32 * k0, M::mul(M::mul(rm[32 * k0], scale), __ldg(wm + 32 * k0)));
	}
}

// --- A1 / A2 on the row pipeline (rowpipe.cuh): many rows, rows of at most
// a few thousand floats, 16-byte aligned.  Same arithmetic in the same order
// as the kernels above; only where the row's elements come from differs.
template <int S>
__global__ void __launch_bounds__(kPipeMaxWarps * 32, 1) k_rmsnorm_pipe(float *o, const float *x, const float *w, int64_t rows, int n, float eps)
{
	extern __shared__ __align__(128) unsigned char smem[];
	using M = F<false>;
	const int W = blockDim.x >> 5;
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const PipeLayout L = pipe_layout(n, 1, W, S);
	const int64_t nw = (int64_t)gridDim.x * W;
	// rows interleaved over the CTAs first: CTA b holds rows b, b + G, b + 2G,
	// ... (every SM within one row of the average), its warp w the ones from
	// b + G w on, every G W
	const int64_t first = (int64_t)warp * gridDim.x + blockIdx.x;
	const float *const src[1] = {x};
	WarpPipe<S, 1> p = pipe_start<S, 1>(smem, L, src, w, n, first, nw, rows);
	const float4 *g4 = reinterpret_cast<const float4 *>(smem);
	bool ok = pipe_wait_gamma(p, smem, L, first, nw, rows);
	const int vpl = n >> 5, n4 = n >> 2;
	const float nf = (float)n;
	for (int64_t row = first; ok && row < rows; row += nw) {
		float *xs = p.slot((int)(p.waited % S), 0);
		if (!p.wait()) {
			ok = false;
			break;
		}
		// pass 1: chain l = elements l + 32k, from shared memory
		float acc = 0.0f;
#pragma unroll 8
		for (int k = 0; k < vpl; ++k) {
			const float v = xs[lane + 32 * k];
			acc = M::fma(v, v, acc);
		}
		const float scale = rms_scale<false>(reduce_chains_4x8<false>(acc), nf, eps);
		// pass 2: (x * scale) * w, float4 per lane, straight to global memory
		const float4 *x4 = reinterpret_cast<const float4 *>(xs);
		float4 *o4 = reinterpret_cast<float4 *>(o + row * n);
		for (int i = lane; i < n4; i += 32) {
			const float4 v = x4[i], g = g4[i];
			st_stream4(o4 + i, make_float4(M::mul(M::mul(v.x, scale), g.x), M::mul(M::mul(v.y, scale), g.y), M::mul(M::mul(v.z, scale), g.z),
			                               M::mul(M::mul(v.w, scale), g.w)));
		}
		__syncwarp(); // every lane is done with the slot before it is refilled
		const int64_t next = row + S * nw;
		if (next < rows)
			p.issue(next, lane == 0);
	}
	if (!ok)
		p.drain();
}

// Launches a row-pipeline kernel: one CTA per SM (at most one per W rows),
// W warps as the shared-memory budget allows.  Returns V7G_ERR_UNSUPPORTED
// when the rows are too long for two warps' slots.
template <typename Kernel, typename... Args>
int launch_pipe(Kernel kernel, int stages, uint64_t &smem_flag, const char *what, int64_t rows, int n, int nin, void *stream, Args... args)
{
	DeviceInfo dev;
	int rc = current_device(&dev);
	if (rc != V7G_OK)
		return rc;
	const int W = pipe_warps_for(n, nin, stages, rows, dev.sm_count);
	if (W == 0)
		return V7G_ERR_UNSUPPORTED;
	if (pipe_allow_smem(kernel, dev.device, smem_flag) != 0)
		return V7G_ERR_UNSUPPORTED;
	const int64_t want = (rows + W - 1) / W;
	const int grid = (int)(want < dev.sm_count ? want : dev.sm_count);
	const uint32_t smem = pipe_layout(n, nin, W, stages).total();
	const cudaError_t launched = launch_kernel(kernel, grid, W * 32, smem, stream, args...);
	return check_launch(what, launched);
}

uint64_t g_smem_rms = 0;
// RMSNorm takes the row pipeline from 257 rows on: measured on B200 at
// n = 2048, back to back over inputs larger than L2, against the
// register-chunk kernel above, 2048 rows 7.9 -> 7.6 us, 4096 rows 14.6 ->
// 12.5 us, 8192 rows 26.5 -> 23.5 us, 16384 rows 48.0 -> 47.0 us; three
// stages beat two and four.  (The fused add on the same pipeline, two 8 KB
// rows a slot: with three slots and four warps per SM faster at 4096 rows
// only -- 25.0 -> 24.4 us -- and slower at 2048 and 8192; with one slot and
// 13 warps slower still against the register-chunk kernel with its float4
// pass 2 -- 4096 rows 24.6 -> 25.8 us, 2048 rows 12.5 -> 16.3 us; it keeps
// the register-chunk kernel.)
constexpr int kRmsPipeStages = 3;

// slots per lane per chunk: as deep as 64 registers allow without spills
constexpr int kRmsChunk = 32;
constexpr int kAddChunk = 16;
// Few rows (a decode step, a single vector) leave the GPU mostly idle and
// the time is the row's own latency: then a deeper chunk without the
// occupancy cap puts a 2048-wide row's loads in flight at once.  Same
// arithmetic in the same order, so results are identical.
constexpr int64_t kFewRows = 1024;
// Up to about one row per SM, a CTA of one warp per row: the rows spread over
// as many SMs (each SM's load pipeline serves one row) instead of eight to
// a CTA on a few SMs.
constexpr int64_t kSpreadRows = 256;
constexpr int kRmsChunkFew = 64;
constexpr int kAddChunkFew = 32;

// `oversubscribe` x the resident CTAs of `block` threads, at most one warp
// per row.
template <typename Kernel, typename... Args>
int launch_rows(Kernel kernel, const char *what, int64_t rows, int oversubscribe, int block, void *stream, Args... args)
{
	DeviceInfo dev;
	int rc = current_device(&dev);
	if (rc != V7G_OK)
		return rc;
	const int warps = block / 32;
	const int64_t want = (rows + warps - 1) / warps;
	const int resident = resident_grid((const void *)kernel, block, 0, want, dev);
	const int grid = (int)(want < (int64_t)oversubscribe * resident ? want : (int64_t)oversubscribe * resident);
	const cudaError_t launched = launch_kernel(kernel, grid, block, 0, stream, args...);
	return check_launch(what, launched);
}

bool row_len_ok(int n) { return n > 0 && n < (1 << 24); }

} // namespace
} // namespace v7g

using namespace v7g;

extern "C" {

int v7g_rmsnorm_rows(float *o, const float *x, const float *w, int64_t rows, int n, float eps, void *stream)
{
	if (!row_len_ok(n) || n % 32 != 0)
		return set_error(V7G_ERR_ARG, "v7g_rmsnorm_rows: n = %d must be a positive multiple of 32 below 2^24", n);
	if (rows < 0)
		return set_error(V7G_ERR_ARG, "v7g_rmsnorm_rows: rows = %lld < 0", (long long)rows);
	if (rows == 0)
		return clear_error();
	if (!o || !x || !w)
		return set_error(V7G_ERR_ARG, "v7g_rmsnorm_rows: NULL pointer");
	if (rows > kSpreadRows && aligned16(o) && aligned16(x) && aligned16(w)) {
		const int rc = launch_pipe(k_rmsnorm_pipe<kRmsPipeStages>, kRmsPipeStages, g_smem_rms, "v7g_rmsnorm_rows", rows, n, 1, stream, o, x, w, rows, n, eps);
		if (rc != V7G_ERR_UNSUPPORTED)
			return rc;
	}
	if (rows <= kSpreadRows)
		return launch_rows(k_rmsnorm_rows<kRmsChunkFew, 1, 32>, "v7g_rmsnorm_rows", rows, 1, 32, stream, o, x, w, rows, n, eps);
	if (rows <= kFewRows)
		return launch_rows(k_rmsnorm_rows<kRmsChunkFew, 1>, "v7g_rmsnorm_rows", rows, 1, kBlock, stream, o, x, w, rows, n, eps);
	return launch_rows(k_rmsnorm_rows<kRmsChunk>, "v7g_rmsnorm_rows", rows, 1, kBlock, stream, o, x, w, rows, n, eps);
}

int v7g_fused_add_rmsnorm_rows(float *o, float *residual, const float *add, const float *w, int64_t rows, int n, float eps, void *stream)
{
	if (!row_len_ok(n) || n % 8 != 0)
		return set_error(V7G_ERR_ARG, "v7g_fused_add_rmsnorm_rows: n = %d must be a positive multiple of 8 below 2^24", n);
	if (rows < 0)
		return set_error(V7G_ERR_ARG, "v7g_fused_add_rmsnorm_rows: rows = %lld < 0", (long long)rows);
	if (rows == 0)
		return clear_error();
	if (!o || !residual || !add || !w)
		return set_error(V7G_ERR_ARG, "v7g_fused_add_rmsnorm_rows: NULL pointer");
	// pass 2 in float4 when the rows allow it
	const bool vec = aligned16(o) && aligned16(residual) && aligned16(w) && n % 4 == 0;
	if (rows <= kSpreadRows)
		return vec ? launch_rows(k_fused_add_rmsnorm_rows<kAddChunkFew, 1, 32, true>, "v7g_fused_add_rmsnorm_rows", rows, 4, 32, stream, o, residual, add, w,
		                         rows, n, eps)
		           : launch_rows(k_fused_add_rmsnorm_rows<kAddChunkFew, 1, 32>, "v7g_fused_add_rmsnorm_rows", rows, 4, 32, stream, o, residual, add, w, rows, n,
		                         eps);
	if (rows <= kFewRows)
		return vec ? launch_rows(k_fused_add_rmsnorm_rows<kAddChunkFew, 1, kBlock, true>, "v7g_fused_add_rmsnorm_rows", rows, 4, kBlock, stream, o, residual,
		                         add, w, rows, n, eps)
		           : launch_rows(k_fused_add_rmsnorm_rows<kAddChunkFew, 1>, "v7g_fused_add_rmsnorm_rows", rows, 4, kBlock, stream, o, residual, add, w, rows,
		                         n, eps);
	// CTAs of two warps: the rows spread over the SMs in finer steps (2048
	// rows 12.4 -> 11.9 us, 16384 rows 88.4 -> 87.6 us against eight-warp CTAs)
	if (vec)
		return launch_rows(k_fused_add_rmsnorm_rows<kAddChunk, kMinBlocks * 4, 64, true>, "v7g_fused_add_rmsnorm_rows", rows, 4, 64, stream, o, residual, add,
		                   w, rows, n, eps);
	return launch_rows(k_fused_add_rmsnorm_rows<kAddChunk>, "v7g_fused_add_rmsnorm_rows", rows, 4, kBlock, stream, o, residual, add, w, rows, n, eps);
}

} // extern "C"

namespace v7g {
// Given-up waits of this unit's row pipelines (added into v7g_pipeline_timeouts).
unsigned int norm_pipe_timeouts() { return rowpipe_timeouts_here(); }
} // namespace v7g
