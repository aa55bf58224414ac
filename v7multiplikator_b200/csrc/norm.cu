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
template <int C, int MINB = kMinBlocks, int BLOCK = kBlock>
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
	if (rows <= kSpreadRows)
		return launch_rows(k_fused_add_rmsnorm_rows<kAddChunkFew, 1, 32>, "v7g_fused_add_rmsnorm_rows", rows, 4, 32, stream, o, residual, add, w, rows, n,
		                   eps);
	if (rows <= kFewRows)
		return launch_rows(k_fused_add_rmsnorm_rows<kAddChunkFew, 1>, "v7g_fused_add_rmsnorm_rows", rows, 4, kBlock, stream, o, residual, add, w, rows,
		                   n, eps);
	return launch_rows(k_fused_add_rmsnorm_rows<kAddChunk>, "v7g_fused_add_rmsnorm_rows", rows, 4, kBlock, stream, o, residual, add, w, rows, n, eps);
}

} // extern "C"
