// swiglu.cu -- elementwise SwiGLU, SwiGLU -> Q8 and Q8 quantisation.
//
// All three stream activations once through registers (HBM-bound, no tensor
// cores: a handful of FLOPs per 8-12 bytes).  The Q8 kernels treat a tensor
// whose rows are a multiple of 64 long as a flat sequence of 64-element
// groups -- codes [rows, n] and scales [rows, n/64] are then simply group g at
// byte 64g and scale slot g -- and give each group to a half-warp: lane L of
// the half holds elements 4L..4L+3 as one float4 (16-byte loads, one 4-byte
// code store per lane).  Rows of other lengths (and unaligned pointers) go
// through a general kernel, one warp per group, that also implements the
// reference's trailing-group rule.
#include <algorithm>

#include "internal.h"
#include "launch.cuh"
#include "q8_fast.cuh"

namespace v7g {
namespace {

constexpr int kBlock = 256;
// group pairs per warp iteration of the flat Q8 kernel
constexpr int kQ8Unroll = 2;

// --- A5  elementwise SwiGLU ---------------------------------------------
// VEC: float4 body over count/4 vectors, the (< 4) trailing elements by the
// first threads of block 0.
template <bool VEC>
__global__ void __launch_bounds__(kBlock) k_swiglu(float *out, const float *gate, const float *up, int64_t count)
{
	kernel_entry();
	const int64_t tid = (int64_t)blockIdx.x * kBlock + threadIdx.x;
	const int64_t nthreads = (int64_t)gridDim.x * kBlock;
	if (VEC) {
		const int64_t n4 = count >> 2;
		const float4 *g4 = reinterpret_cast<const float4 *>(gate);
		const float4 *u4 = reinterpret_cast<const float4 *>(up);
		float4 *o4 = reinterpret_cast<float4 *>(out);
		for (int64_t i = tid; i < n4; i += nthreads)
			st_stream4(o4 + i, v7_swiglu4(ld_stream4(g4 + i), ld_stream4(u4 + i)));
		const int64_t t = (n4 << 2) + tid;
		if (tid < (count & 3))
			out[t] = v7_swiglu(gate[t], up[t]);
	} else {
		for (int64_t i = tid; i < count; i += nthreads)
			out[i] = v7_swiglu(gate[i], up[i]);
	}
}

// --- A6 / A8  Q8 over flat 64-element groups (n % 64 == 0, 16-byte aligned) ---
// A warp iteration covers 2*U consecutive groups: half-warp h takes groups
// base + 2u + h, u < U.  The loads of the warp's next iteration are issued
// before the current one is computed (two register sets used in turn), so
// every warp keeps 4U 16-byte loads in flight through its arithmetic.  SWIGLU
// computes h = swiglu(a, b) in registers first (A8), otherwise h = a (A6).
//
// The kernel is close to its instruction-issue limit at HBM speed, so the
// common case is kept short: per-lane pointers advance by one increment per
// iteration (no 64-bit index arithmetic per access), full iterations carry no
// bounds tests, one vote per iteration decides for all 2U groups whether any
// holds an infinity or NaN, and when none does the scales come in pair
// arithmetic and each code from one rounded product and one rounded sum
// (|h * recip| < 127.5 there, so the reference's saturation never acts).
// Otherwise the general path runs: the exact MAXPS tree where a NaN makes the
// order matter, the IEEE scale for an infinite maximum, clamped codes.
template <int U>
struct Q8Regs {
	float4 x[U], y[U];
};

template <bool SWIGLU, int U>
__device__ __forceinline__ void q8_load(Q8Regs<U> &r, const float4 *pa, const float4 *pb)
{
#pragma unroll
	for (int u = 0; u < U; ++u) {
		r.x[u] = ld_stream4(pa + 32 * u);
		if (SWIGLU)
			r.y[u] = ld_stream4(pb + 32 * u);
	}
}

// Quantises the 2U groups held in r; the group of (u, this half-warp) goes to
// pc + 32u (codes, 16 words per group) and ps + 2u (its scale).
template <bool SWIGLU, int U>
__device__ __forceinline__ void q8_iteration(const Q8Regs<U> &r, uint32_t *pc, float *ps, int lane, int hl)
{
	float4 h[U];
#pragma unroll
	for (int u = 0; u < U; ++u)
		h[u] = SWIGLU ? v7_swiglu4(r.x[u], r.y[u]) : r.x[u];
	uint32_t code[U];
	float scale[U];
	q8_groups_f4<U>(h, lane, code, scale);
#pragma unroll
	for (int u = 0; u < U; ++u) {
		__stcs(pc + 32 * u, code[u]);
		if (hl == 0)
			__stcs(ps + 2 * u, scale[u]);
	}
}

// four CTAs per SM: at most 64 registers a thread
template <bool SWIGLU, int U>
__global__ void __launch_bounds__(kBlock, 4) k_q8_groups(uint32_t *codes, float *scales, const float4 *a, const float4 *b, int64_t ngroups)
{
	kernel_entry();
	const int lane = threadIdx.x & 31;
	const int half = lane >> 4;
	const int hl = lane & 15;
	const int64_t nwarps = ((int64_t)gridDim.x * kBlock) >> 5;
	const int64_t warp = ((int64_t)blockIdx.x * kBlock + threadIdx.x) >> 5;
	const int64_t nfull = ngroups / (2 * U); // iterations with all 2U groups present
	// this lane's element of its first group: group 2U*warp + half, float4 hl
	const int64_t g0 = 2 * U * warp + half;
	const float4 *pa = a + g0 * 16 + hl;
	const float4 *pb = SWIGLU ? b + g0 * 16 + hl : nullptr;
	uint32_t *pc = codes + g0 * 16 + hl;
	float *ps = scales + g0;
	const int64_t step = 2 * U * nwarps; // groups per sweep of all warps
	int64_t it = warp;
	if (it < nfull) {
		Q8Regs<U> r0, r1;
		q8_load<SWIGLU, U>(r0, pa, pb);
		for (;;) {
			// r0 holds iteration `it`
			const bool more = it + nwarps < nfull;
			if (more)
				q8_load<SWIGLU, U>(r1, pa + step * 16, SWIGLU ? pb + step * 16 : nullptr);
			q8_iteration<SWIGLU, U>(r0, pc, ps, lane, hl);
			pa += step * 16;
			if (SWIGLU)
				pb += step * 16;
			pc += step * 16;
			ps += step;
			it += nwarps;
			if (!more)
				break;
			// r1 holds iteration `it`
			const bool more1 = it + nwarps < nfull;
			if (more1)
				q8_load<SWIGLU, U>(r0, pa + step * 16, SWIGLU ? pb + step * 16 : nullptr);
			q8_iteration<SWIGLU, U>(r1, pc, ps, lane, hl);
			pa += step * 16;
			if (SWIGLU)
				pb += step * 16;
			pc += step * 16;
			ps += step;
			it += nwarps;
			if (!more1)
				break;
		}
	}
	// the one partial iteration (fewer than 2U groups left), if any: by the
	// warp whose turn it is, group by group with bounds tests
	if (it == nfull && nfull * 2 * U < ngroups) {
#pragma unroll 1
		for (int u = 0; u < U; ++u) {
			const int64_t g = 2 * U * it + 2 * u + half;
			float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f), y = x;
			if (g < ngroups) {
				x = ld_stream4(a + g * 16 + hl);
				if (SWIGLU)
					y = ld_stream4(b + g * 16 + hl);
			}
			const float4 h = SWIGLU ? v7_swiglu4(x, y) : x;
			float scale, recip;
			q8_scale_fast(group_absmax_f4(h, lane), scale, recip);
			if (g < ngroups) {
				__stcs(codes + g * 16 + hl, q8_codes4_x2(h, recip));
				if (hl == 0)
					__stcs(scales + g, scale);
			}
		}
	}
}

// --- general Q8: any row length, any alignment -----------------------------
// One warp per group (row r, group j); lane l holds elements 64j + l and
// 64j + 32 + l of the row.  A full group follows the vector path's MAXPS tree;
// a trailing group of fewer than 64 elements follows the scalar tail path
// (quantize_kernel.inc:119-152).
template <bool SWIGLU>
__global__ void __launch_bounds__(kBlock) k_q8_general(int8_t *codes, float *scales, const float *a, const float *b, int64_t rows, int n)
{
	kernel_entry();
	using M = F<true>;
	const int lane = threadIdx.x & 31;
	const int64_t nwarps = ((int64_t)gridDim.x * kBlock) >> 5;
	const int groups_per_row = (n + kQ8Group - 1) / kQ8Group;
	const int64_t total = rows * groups_per_row;
	for (int64_t gi = ((int64_t)blockIdx.x * kBlock + threadIdx.x) >> 5; gi < total; gi += nwarps) {
		const int64_t row = gi / groups_per_row;
		const int j = (int)(gi - row * groups_per_row);
		const int r = min(kQ8Group, n - kQ8Group * j);
		const int64_t base = row * n + (int64_t)kQ8Group * j;
		const bool v0 = lane < r, v1 = lane + 32 < r;
		float h0 = 0.0f, h1 = 0.0f;
		if (v0)
			h0 = SWIGLU ? v7_swiglu(a[base + lane], b[base + lane]) : a[base + lane];
		if (v1)
			h1 = SWIGLU ? v7_swiglu(a[base + 32 + lane], b[base + 32 + lane]) : a[base + 32 + lane];
		float scale, recip;
		if (r == kQ8Group) {
			q8_scale(group_absmax_w2(h0, h1, lane), scale, recip);
			codes[base + lane] = (int8_t)(q8_code_bits(M::mul(h0, recip)) & 0xffu);
			codes[base + 32 + lane] = (int8_t)(q8_code_bits(M::mul(h1, recip)) & 0xffu);
		} else {
			q8_scale(tail_absmax_w2(h0, v0, h1, v1), scale, recip);
			if (v0)
				codes[base + lane] = (int8_t)(q8_tail_code_bits(M::mul(h0, recip)) & 0xffu);
			if (v1)
				codes[base + 32 + lane] = (int8_t)(q8_tail_code_bits(M::mul(h1, recip)) & 0xffu);
		}
		if (lane == 0)
			scales[gi] = scale;
	}
}

// `oversubscribe` x the blocks that fit resident at once, at most work_blocks:
// the streaming kernels gain from a few waves of CTAs (measured on B200: 2-4x
// beats 1x by ~3 % on the SwiGLU->Q8 kernel).
template <typename Kernel, typename... Args>
int launch_persistent(Kernel kernel, const char *what, int64_t work_blocks, int oversubscribe, void *stream, Args... args)
{
	DeviceInfo dev;
	int rc = current_device(&dev);
	if (rc != V7G_OK)
		return rc;
	const int resident = resident_grid((const void *)kernel, kBlock, 0, work_blocks, dev);
	const int grid = (int)std::min<int64_t>(work_blocks, (int64_t)resident * oversubscribe);
	const cudaError_t launched = launch_kernel(kernel, grid, kBlock, 0, stream, args...);
	return check_launch(what, launched);
}

int q8_rows(const char *what, int8_t *codes, float *scales, const float *a, const float *b, int64_t rows, int n, void *stream, bool swiglu)
{
	if (rows < 0 || n <= 0)
		return set_error(V7G_ERR_ARG, "%s: rows = %lld, n = %d: need rows >= 0 and n > 0", what, (long long)rows, n);
	if (rows == 0)
		return clear_error();
	if (!codes || !scales || !a || (swiglu && !b))
		return set_error(V7G_ERR_ARG, "%s: NULL pointer", what);
	const bool flat = n % kQ8Group == 0 && aligned16(codes) && aligned16(a) && (!swiglu || aligned16(b));
	if (flat) {
		constexpr int U = kQ8Unroll;
		const int64_t ngroups = rows * (n / kQ8Group);
		const int64_t warps = (ngroups + 2 * U - 1) / (2 * U);
		const int64_t blocks = (warps + kBlock / 32 - 1) / (kBlock / 32);
		uint32_t *c4 = reinterpret_cast<uint32_t *>(codes);
		const float4 *a4 = reinterpret_cast<const float4 *>(a), *b4 = reinterpret_cast<const float4 *>(b);
		if (swiglu) {
			// waves of resident CTAs by size: about eight iterations per warp
			// and wave, two to eight waves (measured on B200, back to back:
			// 2.2 % faster than four waves at 16384 x 12288, 3 % at 1024 rows,
			// never slower at the row shards of 2-8 GPUs)
			DeviceInfo dev;
			const int rc = current_device(&dev);
			if (rc != V7G_OK)
				return rc;
			const int64_t resident = resident_grid((const void *)k_q8_groups<true, U>, kBlock, 0, blocks, dev);
			const int64_t waves = std::min<int64_t>(8, std::max<int64_t>(2, (blocks / resident + 4) / 8));
			return launch_persistent(k_q8_groups<true, U>, what, blocks, (int)waves, stream, c4, scales, a4, b4, ngroups);
		}
		return launch_persistent(k_q8_groups<false, U>, what, blocks, 4, stream, c4, scales, a4, b4, ngroups);
	}
	const int64_t total = rows * ((n + kQ8Group - 1) / kQ8Group);
	const int64_t blocks = (total + kBlock / 32 - 1) / (kBlock / 32);
	if (swiglu)
		return launch_persistent(k_q8_general<true>, what, blocks, 1, stream, codes, scales, a, b, rows, n);
	return launch_persistent(k_q8_general<false>, what, blocks, 1, stream, codes, scales, a, b, rows, n);
}

} // namespace
} // namespace v7g

using namespace v7g;

extern "C" {

int v7g_swiglu(float *out, const float *gate, const float *up, int64_t count, void *stream)
{
	if (count < 0)
		return set_error(V7G_ERR_ARG, "v7g_swiglu: count = %lld < 0", (long long)count);
	if (count == 0)
		return clear_error();
	if (!out || !gate || !up)
		return set_error(V7G_ERR_ARG, "v7g_swiglu: NULL pointer");
	if (aligned16(out) && aligned16(gate) && aligned16(up)) {
		const int64_t blocks = ((count >> 2) + kBlock - 1) / kBlock;
		// up to 64 waves of CTAs, in practice one float4 per thread: the
		// simple stream runs fastest as a one-shot grid (measured on B200:
		// 59.6 us for C4 against 62.9 us at four resident waves)
		return launch_persistent(k_swiglu<true>, "v7g_swiglu", blocks < 1 ? 1 : blocks, 64, stream, out, gate, up, count);
	}
	return launch_persistent(k_swiglu<false>, "v7g_swiglu", (count + kBlock - 1) / kBlock, 1, stream, out, gate, up, count);
}

int v7g_swiglu_q8_rows(int8_t *codes, float *scales, const float *gate, const float *up, int64_t rows, int n, void *stream)
{
	if (n <= 0 || n % kQ8Group != 0)
		return set_error(V7G_ERR_ARG, "v7g_swiglu_q8_rows: n = %d must be a positive multiple of 64", n);
	return q8_rows("v7g_swiglu_q8_rows", codes, scales, gate, up, rows, n, stream, true);
}

int v7g_quantize_rows(int8_t *codes, float *scales, const float *x, int64_t rows, int n, void *stream)
{
	return q8_rows("v7g_quantize_rows", codes, scales, x, nullptr, rows, n, stream, false);
}

} // extern "C"
