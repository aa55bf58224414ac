// gemv.cu -- Q8-weight matrix-vector products: v7d_q8, v7d_swiglu_q8, the
// quantise-then-multiply v7d_q8_fused, and the fp32-activation v7d_swiglu.
//
// Arithmetic of the reference (q8_kernel.inc:22-201, swiglu_q8_kernel.inc:
// 16-286, swiglu_kernel.inc:30-249), reproduced bit for bit:
//   Q8 x Q8: per 64-element group, eight int32 "lane" dots -- lane l covers
//     bytes 4l..4l+3 of the group's low 32 bytes and 4l..4l+3 of its high 32
//     (vpmaddubsw / vpmaddwd / vpaddd); each converted to float (exact), the
//     weight scale times the activation scale rounded once, one fused
//     multiply-add per lane into eight lane accumulators; at the end the
//     HADD_YMM tree (l_j + l_{j+4}, then (t0 + t1) + (t2 + t3)).
//   F32 x Q8 (dual-row path): per element e, w_e converted to float times its
//     group scale (rounded), fused multiply-add with x_e into lane e % 8 of
//     one accumulator; HADD_YMM at the end.
//   SwiGLU epilogue: (sigmoid(g) * g) * u with EVAL_SIGMOID.  FTZ+DAZ
//   throughout (the reference runs these on its dispatched workers).
//
// The lane accumulators are eight independent fp32 chains per output row, so
// the GPU runs one chain per thread: eight threads per row, four rows per
// warp; lane l's dot uses the row's bytes 4l..4l+3 and 32+4l..32+4l+3 of
// every group (dp4a).  The weights are read exactly once: HBM-bound at
// d x n x (1 + 4/64) bytes per matrix.  Three kernels share this arithmetic:
//   k_q8_gemv_stream  weights and scales 16-byte aligned, groups % 4 == 0:
//                     persistent CTAs, producer warps stream activation,
//                     scales and weight chunks by bulk copy into shared
//                     memory rings (the decode-size fast path); a batch of
//                     Q8 activation rows goes in blocks of 2 or 4 rows that
//                     share one weight stream (token blocks);
//   k_q8_gemv_tma     weights aligned but scales not: one producer warp, a
//                     per-CTA ring, the scales read by the consumers;
//   k_q8_gemv         anything else: direct 4-byte loads, kUnroll groups
//                     issued before their arithmetic.
// The entry points pick the first that applies.
#include <algorithm>
#include <atomic>

#include "arith.cuh"
#include "internal.h"
#include "launch.cuh"
#include "pipeline.cuh"
#include "q8.cuh"
#include "q8_fast.cuh"

namespace v7g {
namespace {

constexpr int kBlock = 256;
constexpr int kLanes = 8;                     // HADD_YMM lanes per row
constexpr int kRowsPerBlock = kBlock / kLanes; // 32
constexpr int kUnroll = 8;                    // groups loaded ahead of their arithmetic
constexpr int kMaxN = 65536;                  // activation staged in shared memory

// The weight bytes the reference's vpsignb cannot negate: a -128 weight
// against a negative activation contributes |a| * (-128) there instead of
// a * (-128), i.e. 256 * a more than the true product.  The exporter never
// writes -128 (swiglu_q8_kernel.inc:17-23), so this runs only on inputs
// outside that contract.
__device__ __forceinline__ int neg128_correction(uint32_t a, uint32_t w)
{
	int c = 0;
#pragma unroll
	for (int k = 0; k < 4; ++k) {
		const int ab = (int)(int8_t)(a >> (8 * k));
		const uint32_t wb = (w >> (8 * k)) & 0xffu;
		if (wb == 0x80u && ab < 0)
			c += 256 * ab;
	}
	return c;
}

// Non-zero when a byte of w is 0x80 (-128).
__device__ __forceinline__ uint32_t has_neg128(uint32_t w)
{
	const uint32_t t = w ^ 0x80808080u;
	return (t - 0x01010101u) & ~t & 0x80808080u;
}


// One lane's dot over one group (the low word and the high word) as the
// true products; *flag collects whether a -128 weight byte needs the
// correction, which the callers apply once per batch of groups so that the
// groups' dots stay free of branches.
__device__ __forceinline__ int lane_dot(uint32_t a_lo, uint32_t w_lo, uint32_t a_hi, uint32_t w_hi, uint32_t &flag)
{
	flag |= has_neg128(w_lo) | has_neg128(w_hi);
	return __dp4a((int)a_hi, (int)w_hi, __dp4a((int)a_lo, (int)w_lo, 0));
}

__device__ __forceinline__ int lane_dot_correction(uint32_t a_lo, uint32_t w_lo, uint32_t a_hi, uint32_t w_hi)
{
	return neg128_correction(a_lo, w_lo) + neg128_correction(a_hi, w_hi);
}

// The same, out of line: for loops where it is cold code that would otherwise
// crowd the instruction cache.
static __device__ __noinline__ int lane_dot_correction_call(uint32_t a_lo, uint32_t w_lo, uint32_t a_hi, uint32_t w_hi)
{
	return lane_dot_correction(a_lo, w_lo, a_hi, w_hi);
}

// HADD_YMM over the row's eight lane threads (consecutive lanes of a warp):
// (l_j + l_{j+4}), then (t0 + t1) + (t2 + t3); the sum lands in lane j = 0.
__device__ __forceinline__ float hadd_lanes(float v)
{
	using M = F<true>;
	v = M::add(v, __shfl_xor_sync(0xffffffffu, v, 4));
	v = M::add(v, __shfl_xor_sync(0xffffffffu, v, 1));
	return M::add(v, __shfl_xor_sync(0xffffffffu, v, 2));
}

struct GemvArgs {
	float *out;            // [batch, d]
	const int8_t *xq;      // [batch, n] codes (Q8 activation)
	const float *xs;       // [batch, n/64]
	const float *xf;       // [batch, n] fp32 activation (fused quantise, F32 x Q8)
	const int8_t *wq[2];   // gate (or the only matrix), up: [d, n]
	const float *ws[2];    // [d, n/64]
	int n, d;
	int batch;             // activation rows (the token-block kernels)
};

// Quantise the CTA's activation row into shared memory with v7d_quantize's
// rules (quantize_kernel.inc:43-106): half a warp per 64-element group, one
// float4 per lane; `nthreads` (a multiple of 32) threads take part.  SHARED:
// x is a 16-byte aligned copy in shared memory (plain loads), else global.
// Groups [gbeg, gend) only when gend >= 0 (x, sq, ss still indexed from group 0).
// IL: the codes land in the interleaved layout of the streaming kernel (word
// 2l of a group = word l, word 2l + 1 = word 8 + l).  U: group pairs per
// warp loaded before any is processed (one latency per U, and compact code).
template <bool SHARED = false, bool IL = false, int U = 4>
__device__ __noinline__ void stage_quantized(const float *x, int n, uint32_t *sq, float *ss, int nthreads = kBlock, int gbeg = 0, int gend = -1)
{
	const int lane = threadIdx.x & 31, half = lane >> 4, hl = lane & 15;
	const int groups = gend >= 0 ? gend : n / kQ8Group;
	const int step = (nthreads / 32) * 2;
	const bool vec = SHARED || (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
	for (int g0 = gbeg + (threadIdx.x >> 5) * 2; g0 < groups; g0 += U * step) {
		float4 h[U];
#pragma unroll
		for (int u = 0; u < U; ++u) {
			const int g = g0 + u * step + half;
			h[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
			if (g < groups) {
				const float *p = x + (int64_t)g * kQ8Group + 4 * hl;
				if (SHARED)
					h[u] = *reinterpret_cast<const float4 *>(p);
				else
					h[u] = vec ? __ldg(reinterpret_cast<const float4 *>(p)) : make_float4(__ldg(p), __ldg(p + 1), __ldg(p + 2), __ldg(p + 3));
			}
		}
		uint32_t code[U];
		float scale[U];
		q8_groups_f4<U>(h, lane, code, scale); // groups past the end hold zeros: harmless
#pragma unroll
		for (int u = 0; u < U; ++u) {
			const int g = g0 + u * step + half;
			if (g < groups) {
				sq[g * 16 + (IL ? (hl < 8 ? 2 * hl : 2 * hl - 15) : hl)] = code[u];
				if (hl == 0)
					ss[g] = scale[u];
			}
		}
	}
}

// MODE 0: v7d_q8 (one matrix); 1: v7d_swiglu_q8 (gate, up, SwiGLU epilogue).
// FUSED: the activation arrives as fp32 and is quantised here first.
template <int MODE, bool FUSED>
__global__ void __launch_bounds__(kBlock) k_q8_gemv(GemvArgs p)
{
	kernel_entry();
	using M = F<true>;
	constexpr int NM = MODE == 1 ? 2 : 1;
	extern __shared__ __align__(128) unsigned char smem[];
	const int n = p.n, groups = n / kQ8Group;
	uint32_t *sq = reinterpret_cast<uint32_t *>(smem);
	float *ss = reinterpret_cast<float *>(smem + n);
	const int64_t b = blockIdx.y;
	if (FUSED) {
		stage_quantized(p.xf + b * n, n, sq, ss);
	} else {
		const uint4 *src = reinterpret_cast<const uint4 *>(p.xq + b * n);
		for (int i = threadIdx.x; i < n / 16; i += kBlock)
			reinterpret_cast<uint4 *>(smem)[i] = __ldg(src + i);
		for (int i = threadIdx.x; i < groups; i += kBlock)
			ss[i] = __ldg(p.xs + b * groups + i);
	}
	__syncthreads();
	const int l = threadIdx.x & (kLanes - 1);
	// rows past d compute nothing but stay for the lane shuffles
	const int64_t row_raw = (int64_t)blockIdx.x * kRowsPerBlock + (threadIdx.x >> 3);
	const bool valid = row_raw < p.d;
	const int64_t row = valid ? row_raw : 0;
	const int gend = valid ? groups : 0;
	const uint32_t *w[NM];
	const float *s[NM];
#pragma unroll
	for (int m = 0; m < NM; ++m) {
		w[m] = reinterpret_cast<const uint32_t *>(p.wq[m] + row * n) + l;
		s[m] = p.ws[m] + row * groups;
	}
	float acc[NM];
#pragma unroll
	for (int m = 0; m < NM; ++m)
		acc[m] = 0.0f;
	for (int g0 = 0; g0 < gend; g0 += kUnroll) {
		uint32_t lo[NM][kUnroll], hi[NM][kUnroll];
		float sc[NM][kUnroll];
#pragma unroll
		for (int u = 0; u < kUnroll; ++u)
			if (g0 + u < gend) {
#pragma unroll
				for (int m = 0; m < NM; ++m) {
					lo[m][u] = __ldcs(w[m] + (g0 + u) * 16);
					hi[m][u] = __ldcs(w[m] + (g0 + u) * 16 + 8);
					sc[m][u] = __ldg(s[m] + g0 + u);
				}
			}
		int dots[NM][kUnroll];
		uint32_t alo[kUnroll], ahi[kUnroll];
		uint32_t flag = 0;
#pragma unroll
		for (int u = 0; u < kUnroll; ++u)
			if (g0 + u < gend) {
				const int g = g0 + u;
				alo[u] = sq[g * 16 + l];
				ahi[u] = sq[g * 16 + 8 + l];
#pragma unroll
				for (int m = 0; m < NM; ++m)
					dots[m][u] = lane_dot(alo[u], lo[m][u], ahi[u], hi[m][u], flag);
			}
		if (flag) {
#pragma unroll
			for (int u = 0; u < kUnroll; ++u)
				if (g0 + u < gend)
#pragma unroll
					for (int m = 0; m < NM; ++m)
						dots[m][u] += lane_dot_correction(alo[u], lo[m][u], ahi[u], hi[m][u]);
		}
#pragma unroll
		for (int u = 0; u < kUnroll; ++u)
			if (g0 + u < gend) {
				const float xsg = ss[g0 + u];
#pragma unroll
				for (int m = 0; m < NM; ++m)
					acc[m] = M::fma((float)dots[m][u], M::mul(sc[m][u], xsg), acc[m]);
			}
	}
	float r[NM];
#pragma unroll
	for (int m = 0; m < NM; ++m)
		r[m] = hadd_lanes(acc[m]);
	if (l == 0 && valid)
		p.out[b * p.d + row] = MODE == 1 ? v7_swiglu(r[0], r[1]) : r[0];
}

// Wait-bound events of the pipelined kernels (device word, read by
// v7g_pipeline_timeouts); 0 in every correct run.
__device__ unsigned int g_pipeline_timeouts;

// ---- pipelined Q8 x Q8 GEMV ------------------------------------------------
// The arithmetic of k_q8_gemv with the weights streamed through shared
// memory: a CTA owns R consecutive rows; one producer thread issues 1-D bulk
// copies of kChunkGroups groups (1 KB) of every row and matrix per stage
// into a ring of `stages` stages (transaction-counting mbarriers), the R x 8
// consumer threads (one per row lane, as in k_q8_gemv) take the words of
// their lane from shared memory.  Tens of KB stay in flight per SM whatever d
// is, so small matrices stream near HBM speed too.
constexpr int kChunkGroups = 16;
// A row's slot in a stage: the 1024 bytes of its chunk and 32 bytes of
// padding, so the four rows a warp reads start 8 banks apart.
constexpr int kRowSlot = kChunkGroups * kQ8Group + 32;
// The same padding for a chunk of cg groups (cg even: rows stay 8 banks apart).
__host__ __device__ constexpr int row_slot(int cg) { return cg * kQ8Group + 32; }

// The chains of one row lane over the gk (<= G) groups of a stage: all dots
// first (no branch between groups), the rare -128 correction once, then the
// fused multiply-adds in group order.  st: the row's slot of matrix 0 (matrix
// m at + m * R slots); a: activation words of the first group; cs: the row's
// combined scales (weight scale times activation scale) from the first group
// (matrix m at + m * R * sstride).
template <int NM, int R, int G>
__device__ __forceinline__ void chunk_chains(float (&acc)[NM], const uint32_t *st, const uint32_t *a, const float *cs, int sstride, int l, int gk)
{
	using M = F<true>;
	constexpr int SB = 4; // groups per batch: bounds the registers the dots hold
#pragma unroll 1
	for (int b0 = 0; b0 < G; b0 += SB) {
		if (b0 >= gk)
			break;
		int dots[NM][SB];
		uint32_t flag = 0;
#pragma unroll
		for (int j = 0; j < SB; ++j)
			if (b0 + j < gk)
#pragma unroll
				for (int m = 0; m < NM; ++m) {
					const uint32_t *wr = st + m * R * (kRowSlot / 4) + (b0 + j) * 16;
					dots[m][j] = lane_dot(a[(b0 + j) * 16 + l], wr[l], a[(b0 + j) * 16 + 8 + l], wr[8 + l], flag);
				}
		if (flag) {
#pragma unroll
			for (int j = 0; j < SB; ++j)
				if (b0 + j < gk)
#pragma unroll
					for (int m = 0; m < NM; ++m) {
						const uint32_t *wr = st + m * R * (kRowSlot / 4) + (b0 + j) * 16;
						dots[m][j] += lane_dot_correction(a[(b0 + j) * 16 + l], wr[l], a[(b0 + j) * 16 + 8 + l], wr[8 + l]);
					}
		}
#pragma unroll
		for (int j = 0; j < SB; ++j)
			if (b0 + j < gk)
#pragma unroll
				for (int m = 0; m < NM; ++m)
					acc[m] = M::fma((float)dots[m][j], cs[m * R * sstride + b0 + j], acc[m]);
	}
}

// fp32 activation x Q8 weights over the gk groups of a stage for row lane l
// (elements e = l mod 8), gate and up as the two halves of a pair: the
// weight byte to float by placing it in the mantissa of 2^23 + 128 and
// subtracting (exact), times its group scale (rounded), fused multiply-add
// with x_e -- the dual-row arithmetic of swiglu_kernel.inc:30-47.  The lane's
// byte of step k is byte 8k + l of the group, read on its own (one shared
// load and one logic op per byte: (u ^ 0x80) | 0x4B000000).  st: the row's
// gate slot (up at + R slots); xl: the lane's activations from the first
// group, 8 per group; sw: the row's gate scales (up at + R * sstride).
template <int R, int CG = kChunkGroups>
__device__ __forceinline__ void chunk_f32(float (&acc)[2], const uint32_t *st, const float *xl, const float *sw, int sstride, int l, int gk)
{
	const float2 bias = splat2(-8388736.0f); // -(2^23 + 128)
	float2 a = make_float2(acc[0], acc[1]);
	const unsigned char *stg = reinterpret_cast<const unsigned char *>(st) + l;
	const unsigned char *stu = stg + R * row_slot(CG);
#pragma unroll 2
	for (int gi = 0; gi < gk; ++gi) {
		const float4 x0 = *reinterpret_cast<const float4 *>(xl + gi * 8);
		const float4 x1 = *reinterpret_cast<const float4 *>(xl + gi * 8 + 4);
		const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
		const float2 sc = make_float2(sw[gi], sw[R * sstride + gi]);
#pragma unroll
		for (int k = 0; k < 8; ++k) {
			const uint32_t gb = stg[gi * kQ8Group + 8 * k], ub = stu[gi * kQ8Group + 8 * k];
			const float2 raw = make_float2(__uint_as_float((gb ^ 0x80u) | 0x4B000000u), __uint_as_float((ub ^ 0x80u) | 0x4B000000u));
			a = fma2(splat2(xv[k]), mul2(add2(raw, bias), sc), a);
		}
	}
	acc[0] = a.x;
	acc[1] = a.y;
}

// MODE 0: v7d_q8, 1: v7d_swiglu_q8, 2: v7d_swiglu (fp32 activation; the
// activation is staged transposed, lane-major, instead of as codes).
template <int MODE, bool FUSED, int R>
__global__ void __launch_bounds__(R * kLanes + 32, 2) k_q8_gemv_tma(GemvArgs p, int stages)
{
	kernel_entry();
	using M = F<true>;
	constexpr int NM = MODE == 0 ? 1 : 2;
	constexpr int kConsumers = R * kLanes;
	constexpr int kStageBytes = NM * R * kRowSlot;
	extern __shared__ __align__(128) unsigned char smem[];
	const int n = p.n, groups = n / kQ8Group;
	const int nchunks = (groups + kChunkGroups - 1) / kChunkGroups;
	const int64_t row0 = (int64_t)blockIdx.x * R;
	const int rows = (int)min((int64_t)R, p.d - row0);
	// layout: stages | activation codes [n] and scales [groups] (MODE 2: the
	// fp32 activation, lane-major [8][xstride]) | weight or combined scales
	// [NM][R][groups + 1] | full[stages] | empty[stages]
	const int sstride = groups + 1; // odd row stride: the warp's four rows hit four banks
	const int xstride = groups * 8 + 4; // MODE 2: padded so the 8 lanes' rows start 4 banks apart
	unsigned char *ring = smem;
	uint32_t *sq = reinterpret_cast<uint32_t *>(smem + (size_t)stages * kStageBytes);
	float *xt = reinterpret_cast<float *>(sq);
	float *ss = reinterpret_cast<float *>(reinterpret_cast<unsigned char *>(sq) + (MODE == 2 ? 32 * xstride : n));
	float *sws = ss + (MODE == 2 ? 0 : groups);
	uint64_t *full = reinterpret_cast<uint64_t *>(sws + NM * R * sstride + ((NM * R * sstride + (MODE == 2 ? 0 : groups)) & 1));
	uint64_t *empty = full + stages;
	const int64_t b = blockIdx.y;
	if (threadIdx.x == 0) {
		for (int s = 0; s < stages; ++s) {
			mbar_init(full + s, 1);
			mbar_init(empty + s, kConsumers / 32);
		}
		mbar_init_fence();
	}
	__syncthreads();
	if (threadIdx.x >= kConsumers) {
		// producer warp: lane 0 waits for the slot and posts the byte count,
		// then every lane issues one row's copy (NM * R <= 32)
		const int lane = threadIdx.x & 31;
		for (int k = 0; k < nchunks; ++k) {
			const int s = k % stages;
			bool ok = true;
			if (k >= stages && lane == 0)
				ok = mbar_wait(empty + s, ((k / stages) - 1) & 1, &g_pipeline_timeouts);
			if (!__shfl_sync(0xffffffffu, ok, 0))
				break;
			const int g0 = k * kChunkGroups;
			const int gk = min(kChunkGroups, groups - g0);
			const uint32_t bytes = (uint32_t)(gk * kQ8Group);
			if (lane == 0)
				mbar_arrive_expect_tx(full + s, bytes * NM * rows);
			__syncwarp();
			if (lane < NM * rows) {
				const int m = lane / rows, r = lane - m * rows;
				// a select, not p.wq[m]: a runtime index into the parameter
				// array would copy it to local memory
				const int8_t *wm = m == 0 ? p.wq[0] : p.wq[NM - 1];
				bulk_copy_g2s(ring + (size_t)s * kStageBytes + (m * R + r) * kRowSlot, wm + (row0 + r) * n + (int64_t)g0 * kQ8Group,
				              bytes, full + s);
			}
		}
		// leave only once the copies of the last stages have landed
		if (lane == 0)
			for (int k = max(0, nchunks - stages); k < nchunks; ++k)
				if (!mbar_wait(full + k % stages, (k / stages) & 1, &g_pipeline_timeouts))
					break;
		return;
	}
	// consumers: stage the activation and the weight scales, then the chains
	if (MODE == 2) {
		const float *xb = p.xf + b * n;
		for (int i = threadIdx.x; i < n; i += kConsumers)
			xt[(i & 7) * xstride + (i >> 6) * 8 + ((i >> 3) & 7)] = __ldg(xb + i);
	} else if (FUSED) {
		stage_quantized(p.xf + b * n, n, sq, ss, kConsumers);
	} else {
		const uint4 *src = reinterpret_cast<const uint4 *>(p.xq + b * n);
		for (int i = threadIdx.x; i < n / 16; i += kConsumers)
			reinterpret_cast<uint4 *>(sq)[i] = __ldg(src + i);
		for (int i = threadIdx.x; i < groups; i += kConsumers)
			ss[i] = __ldg(p.xs + b * groups + i);
	}
	// raw weight scales now (their loads overlap the activation's), each
	// thread's entries turned into combined scales -- weight scale x
	// activation scale, rounded once as the reference's vmulps -- once the
	// activation scales are in place
	for (int m = 0; m < NM; ++m)
		for (int i = threadIdx.x; i < rows * groups; i += kConsumers)
			sws[(m * R + i / groups) * sstride + i % groups] = __ldg(p.ws[m] + row0 * groups + i);
	named_sync(1, kConsumers);
	if (MODE != 2) {
		for (int m = 0; m < NM; ++m)
			for (int i = threadIdx.x; i < rows * groups; i += kConsumers) {
				float *c = sws + (m * R + i / groups) * sstride + i % groups;
				*c = M::mul(*c, ss[i % groups]);
			}
		named_sync(1, kConsumers);
	}
	const int r = threadIdx.x >> 3, l = threadIdx.x & (kLanes - 1);
	const bool valid = r < rows;
	float acc[NM];
#pragma unroll
	for (int m = 0; m < NM; ++m)
		acc[m] = 0.0f;
	bool ok = true;
	for (int k = 0; k < nchunks; ++k) {
		const int s = k % stages;
		// the warp leaves together if any lane's wait ran out
		if (!__all_sync(0xffffffffu, mbar_wait(full + s, (k / stages) & 1, &g_pipeline_timeouts))) {
			ok = false;
			break;
		}
		const int g0 = k * kChunkGroups;
		const int gk = min(kChunkGroups, groups - g0);
		if (valid) {
			const uint32_t *st = reinterpret_cast<const uint32_t *>(ring + (size_t)s * kStageBytes) + r * (kRowSlot / 4);
			const float *cs = sws + r * sstride + g0;
			if constexpr (MODE == 2)
				chunk_f32<R>(acc, st, xt + l * xstride + g0 * 8, cs, sstride, l, gk);
			else if (gk == kChunkGroups)
				chunk_chains<NM, R, kChunkGroups>(acc, st, sq + g0 * 16, cs, sstride, l, kChunkGroups);
			else
				chunk_chains<NM, R, kChunkGroups>(acc, st, sq + g0 * 16, cs, sstride, l, gk);
		}
		__syncwarp();
		if ((threadIdx.x & 31) == 0)
			mbar_arrive(empty + s);
	}
	float res[NM];
#pragma unroll
	for (int m = 0; m < NM; ++m)
		res[m] = hadd_lanes(acc[m]);
	if (ok && valid && l == 0)
		p.out[b * p.d + row0 + r] = MODE == 0 ? res[0] : v7_swiglu(res[0], res[NM - 1]);
}

// ---- streaming Q8 GEMV -------------------------------------------------------
// The arithmetic of k_q8_gemv once more, organised for HBM: a CTA (two per
// SM, or one with twice the ring when there are no more row blocks than SMs)
// walks the row blocks rb = blockIdx.x, + gridDim.x, ... and its P producer
// warps stream, in order and without draining between row blocks:
//   once      the activation (codes and scales, or the fp32 row) -- ahead of
//             every weight byte, so the consumers' prologue is one latency;
//   per block its weight scales, one bulk copy per matrix (the block's rows
//             are contiguous) into a two-slot ring;
//   per chunk the block's CG groups of every row and matrix into a ring of
//             up to kMaxStages stages (kMaxStagesOne for the one-matrix
//             product: with fewer chunks in flight the first ones land
//             sooner, and its consumers, which are the slower side at
//             decode sizes, start sooner -- 6.98 -> 6.80 us at d = 2048,
//             n = 8192, where all four chunks of a block fitted before;
//             kMaxStagesFused for its fused form, whose consumers first
//             quantise the activation: 7.21 us with three, 6.96 with four).
// The consumers re-lay the activation codes so that a lane's two words of a
// group are adjacent (one 8-byte load), and form the combined scale (weight
// scale x activation scale, rounded once as the reference's vmulps) as they
// go.  Requires every weight and scale pointer 16-byte aligned and
// groups % 4 == 0 (16-byte scale rows).
constexpr int kMaxStages = 8;
constexpr int kMaxStagesOne = 3;
constexpr int kMaxStagesFused = 4;

// The lane's two activation words of group g in the streaming kernel's
// interleaved layout (word 2l = word l of the group, 2l + 1 = word 8 + l).
__device__ __forceinline__ uint2 act_words(const uint32_t *a, int g, int l) { return reinterpret_cast<const uint2 *>(a)[g * 8 + l]; }

// One batch of SB groups of one matrix for one token: the lane dots, then
// the chain.  CMB: wsr holds the combined scales (weight scale x activation
// scale, formed once per row block by the kernel) and xsc is unused; else
// the combined scale is formed here per group.  The one-token kernels keep
// this form: the token-block form below with NB = 1 measured about 1 %
// slower at the decode shapes.
// EXACT: a group holding a -128 weight byte gets the reference's product
// (lane_dot_correction).  Otherwise the dots are the true products and the
// returned word is non-zero when a weight byte of the batch is -128: per
// word the zero-byte test of w ^ 0x80808080 ((t - 0x01010101) & ~t, nonzero
// in bit 7 of some byte exactly when a byte of t is zero), the groups' tests
// OR-ed as a tree, not as one dependent chain, and masked once.
template <bool EXACT, bool FULL, bool CMB, int R, int SB, int CG>
__device__ __forceinline__ uint32_t batch_chain1_one(float &acc, const uint32_t *st, const uint32_t *a, const float *wsr, const float *xsc, int l, int b0, int gk)
{
	using M = F<true>;
	int dots[SB];
	uint32_t f[SB];
#pragma unroll
	for (int j = 0; j < SB; ++j) {
		f[j] = 0;
		if (FULL || b0 + j < gk) {
			const uint2 av = act_words(a, b0 + j, l);
			const uint32_t *wr = st + (b0 + j) * 16;
			const uint32_t wlo = wr[l], whi = wr[8 + l];
			dots[j] = __dp4a((int)av.y, (int)whi, __dp4a((int)av.x, (int)wlo, 0));
			if (EXACT) {
				if (has_neg128(wlo) | has_neg128(whi))
					dots[j] += lane_dot_correction_call(av.x, wlo, av.y, whi);
			} else {
				const uint32_t tlo = wlo ^ 0x80808080u, thi = whi ^ 0x80808080u;
				f[j] = ((tlo - 0x01010101u) & ~tlo) | ((thi - 0x01010101u) & ~thi);
			}
		}
	}
	uint32_t flag = 0;
	if (!EXACT) {
#pragma unroll
		for (int w = SB / 2; w >= 1; w /= 2)
#pragma unroll
			for (int j = 0; j < w; ++j)
				f[j] |= f[j + w];
		flag = f[0] & 0x80808080u;
	}
#pragma unroll
	for (int q = 0; q < SB / 4; ++q) {
		const float4 w4 = *reinterpret_cast<const float4 *>(wsr + b0 + 4 * q);
		float cv[4] = {w4.x, w4.y, w4.z, w4.w};
		if (!CMB) {
			const float4 x4 = *reinterpret_cast<const float4 *>(xsc + b0 + 4 * q);
			cv[0] = M::mul(w4.x, x4.x), cv[1] = M::mul(w4.y, x4.y), cv[2] = M::mul(w4.z, x4.z), cv[3] = M::mul(w4.w, x4.w);
		}
#pragma unroll
		for (int u = 0; u < 4; ++u)
			if (FULL || b0 + 4 * q + u < gk)
				acc = M::fma((float)dots[4 * q + u], cv[u], acc);
	}
	return flag;
}

// The chain of one chunk of one matrix (gk groups of the stage's row; FULL:
// gk == CG, so no group needs a bound check).  The fast pass takes the true
// products and tests the weights on the side; if a weight byte of the chunk
// was -128 (outside the exporter's contract), the chunk runs again from the
// accumulator it started with, with the reference's products.  Keeping the
// test's outcome out of the batch loop lets the chain run without waiting on
// it: measured 7.36 -> 6.98 us at d = 2048, n = 8192 against a per-batch
// branch on a serially OR-ed flag.
template <int R, int SB, int CG, bool FULL, bool CMB>
__device__ __forceinline__ void chunk_chain1_one(float &acc, const uint32_t *st, const uint32_t *a, const float *wsr, const float *xsc, int l, int gk)
{
	static_assert(SB % 4 == 0 && CG % SB == 0 && (SB & (SB - 1)) == 0, "batches of whole float4 scale words, a power-of-two tree");
	const int nb = FULL ? CG / SB : (gk + SB - 1) / SB;
	const float acc0 = acc;
	uint32_t flag = 0;
#pragma unroll 1
	for (int k = 0; k < nb; ++k)
		flag |= batch_chain1_one<false, FULL, CMB, R, SB, CG>(acc, st, a, wsr, xsc, l, k * SB, gk);
	if (flag) { // cold
		acc = acc0;
#pragma unroll 1
		for (int k = 0; k < nb; ++k)
			batch_chain1_one<true, FULL, CMB, R, SB, CG>(acc, st, a, wsr, xsc, l, k * SB, gk);
	}
}

// One batch of SB groups of one matrix for NB tokens (activations a + t *
// astride words, their scales xsc + t * sstride): the weight words loaded
// and tested once, each token's lane dots, then each token's chain.
// EXACT: a group holding a -128 weight byte gets the reference's product
// (lane_dot_correction).  Otherwise the dots are the true products and the
// returned word is non-zero when a weight byte of the batch is -128: per
// word the zero-byte test of w ^ 0x80808080 ((t - 0x01010101) & ~t, nonzero
// in bit 7 of some byte exactly when a byte of t is zero), the groups' tests
// OR-ed as a tree, not as one dependent chain, and masked once.
template <bool EXACT, bool FULL, int NB, int SB, int CG>
__device__ __forceinline__ uint32_t batch_chain1(float (&acc)[NB], const uint32_t *st, const uint32_t *a, int astride, const float *wsr, const float *xsc,
                                                 int sstride, int l, int b0, int gk)
{
	using M = F<true>;
	int dots[NB][SB];
	uint32_t f[SB];
#pragma unroll
	for (int j = 0; j < SB; ++j) {
		f[j] = 0;
		if (FULL || b0 + j < gk) {
			const uint32_t *wr = st + (b0 + j) * 16;
			const uint32_t wlo = wr[l], whi = wr[8 + l];
			bool neg = false;
			if (EXACT)
				neg = (has_neg128(wlo) | has_neg128(whi)) != 0;
			else {
				const uint32_t tlo = wlo ^ 0x80808080u, thi = whi ^ 0x80808080u;
				f[j] = ((tlo - 0x01010101u) & ~tlo) | ((thi - 0x01010101u) & ~thi);
			}
#pragma unroll
			for (int t = 0; t < NB; ++t) {
				const uint2 av = act_words(a + t * astride, b0 + j, l);
				dots[t][j] = __dp4a((int)av.y, (int)whi, __dp4a((int)av.x, (int)wlo, 0));
				if (EXACT && neg)
					dots[t][j] += lane_dot_correction_call(av.x, wlo, av.y, whi);
			}
		}
	}
	uint32_t flag = 0;
	if (!EXACT) {
#pragma unroll
		for (int w = SB / 2; w >= 1; w /= 2)
#pragma unroll
			for (int j = 0; j < w; ++j)
				f[j] |= f[j + w];
		flag = f[0] & 0x80808080u;
	}
#pragma unroll
	for (int q = 0; q < SB / 4; ++q) {
		const float4 w4 = *reinterpret_cast<const float4 *>(wsr + b0 + 4 * q);
		const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
		for (int t = 0; t < NB; ++t) {
			const float4 x4 = *reinterpret_cast<const float4 *>(xsc + t * sstride + b0 + 4 * q);
			const float xv[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
			for (int u = 0; u < 4; ++u)
				if (FULL || b0 + 4 * q + u < gk)
					acc[t] = M::fma((float)dots[t][4 * q + u], M::mul(wv[u], xv[u]), acc[t]);
		}
	}
	return flag;
}

// The chains of one chunk of one matrix for NB tokens (gk groups of the
// stage's row; FULL: gk == CG, so no group needs a bound check).  The fast
// pass takes the true products and tests the weights on the side; if a
// weight byte of the chunk was -128 (outside the exporter's contract), the
// chunk runs again from the accumulators it started with, with the
// reference's products.  Keeping the test's outcome out of the batch loop
// lets the chains run without waiting on it: measured 7.36 -> 6.98 us at
// d = 2048, n = 8192 against a per-batch branch on a serially OR-ed flag.
template <int NB, int SB, int CG, bool FULL>
__device__ __forceinline__ void chunk_chain1(float (&acc)[NB], const uint32_t *st, const uint32_t *a, int astride, const float *wsr, const float *xsc, int sstride,
                                             int l, int gk)
{
	static_assert(SB % 4 == 0 && CG % SB == 0 && (SB & (SB - 1)) == 0, "batches of whole float4 scale words, a power-of-two tree");
	const int nb = FULL ? CG / SB : (gk + SB - 1) / SB;
	float acc0[NB];
#pragma unroll
	for (int t = 0; t < NB; ++t)
		acc0[t] = acc[t];
	uint32_t flag = 0;
#pragma unroll 1
	for (int k = 0; k < nb; ++k)
		flag |= batch_chain1<false, FULL, NB, SB, CG>(acc, st, a, astride, wsr, xsc, sstride, l, k * SB, gk);
	if (flag) { // cold
#pragma unroll
		for (int t = 0; t < NB; ++t)
			acc[t] = acc0[t];
#pragma unroll 1
		for (int k = 0; k < nb; ++k)
			batch_chain1<true, FULL, NB, SB, CG>(acc, st, a, astride, wsr, xsc, sstride, l, k * SB, gk);
	}
}

// The chains of one chunk of NM matrices (the SwiGLU pair) for NB tokens:
// per batch of SB groups the dots of both matrices, the -128 test folded
// into them, the correction (when a byte was -128) before the chains.  With
// two matrices this per-batch form measured faster than chunk_chain1's
// deferred one (more registers live across the chunk there).
template <int NM, int NB, int R, int SB = 8, int CG = kChunkGroups>
__device__ __forceinline__ void chunk_chains_ws(float (&acc)[NM][NB], const uint32_t *st, const uint32_t *a, int astride, const float *wsr, int mstride,
                                                const float *xsc, int sstride, int l, int gk)
{
	using M = F<true>;
	static_assert(SB % 4 == 0 && CG % SB == 0, "batches of whole float4 scale words");
	constexpr int kSlotWords = row_slot(CG) / 4;
#pragma unroll 1
	for (int b0 = 0; b0 < CG; b0 += SB) {
		if (b0 >= gk)
			break;
		int dots[NM][NB][SB];
		uint32_t flag = 0;
#pragma unroll
		for (int j = 0; j < SB; ++j)
			if (b0 + j < gk) {
				uint2 av[NB];
#pragma unroll
				for (int t = 0; t < NB; ++t)
					av[t] = act_words(a + t * astride, b0 + j, l);
#pragma unroll
				for (int m = 0; m < NM; ++m) {
					const uint32_t *wr = st + m * R * kSlotWords + (b0 + j) * 16;
#pragma unroll
					for (int t = 0; t < NB; ++t)
						dots[m][t][j] = lane_dot(av[t].x, wr[l], av[t].y, wr[8 + l], flag);
				}
			}
		if (flag) { // cold: the exporter never writes -128
#pragma unroll
			for (int j = 0; j < SB; ++j)
				if (b0 + j < gk) {
#pragma unroll
					for (int m = 0; m < NM; ++m) {
						const uint32_t *wr = st + m * R * kSlotWords + (b0 + j) * 16;
#pragma unroll
						for (int t = 0; t < NB; ++t) {
							const uint2 av = act_words(a + t * astride, b0 + j, l);
							dots[m][t][j] += lane_dot_correction_call(av.x, wr[l], av.y, wr[8 + l]);
						}
					}
				}
		}
#pragma unroll
		for (int t = 0; t < NB; ++t) {
			float xv[SB];
#pragma unroll
			for (int q = 0; q < SB / 4; ++q) {
				const float4 x4 = *reinterpret_cast<const float4 *>(xsc + t * sstride + b0 + 4 * q);
				xv[4 * q] = x4.x, xv[4 * q + 1] = x4.y, xv[4 * q + 2] = x4.z, xv[4 * q + 3] = x4.w;
			}
#pragma unroll
			for (int m = 0; m < NM; ++m) {
				float wv[SB];
#pragma unroll
				for (int q = 0; q < SB / 4; ++q) {
					const float4 w4 = *reinterpret_cast<const float4 *>(wsr + m * mstride + b0 + 4 * q);
					wv[4 * q] = w4.x, wv[4 * q + 1] = w4.y, wv[4 * q + 2] = w4.z, wv[4 * q + 3] = w4.w;
				}
#pragma unroll
				for (int j = 0; j < SB; ++j)
					if (b0 + j < gk)
						acc[m][t] = M::fma((float)dots[m][t][j], M::mul(wv[j], xv[j]), acc[m][t]);
			}
		}
	}
}

struct StreamLayout {
	int stages;
	bool xstaged;  // the fp32 activation arrives by bulk copy (FUSED, MODE 2)
	size_t smem;
};

// Shared memory: ring [stages][NM][R] row slots | weight-scale slots
// [2][NM][R * groups] + 16 | activation: codes [n] + scales [groups + 16]
// (MODE 2: fp32 lane-major [8][xstride]) | fp32 staging [n] when xstaged |
// barriers full[stages], empty[stages], sfull[2], sempty[2], pro.
__host__ __device__ inline size_t stream_fixed(int mode, int rows_per_block, int n, int tokens = 1)
{
	const int nm = mode == 0 ? 1 : 2;
	const size_t groups = (size_t)n / kQ8Group;
	const size_t slots = 4 * (2 * (size_t)nm * rows_per_block * groups + 16);
	const size_t act = mode == 2 ? 32 * (groups * 8 + 4) : (size_t)tokens * ((size_t)n + 4 * (groups + 16));
	return slots + act;
}

// Consumer threads of a row block of R rows: eight a row, rounded up to whole
// warps (the threads of rows R.. of the last warp compute nothing).
__host__ __device__ constexpr int stream_consumers(int rows_per_block) { return (rows_per_block * kLanes + 31) / 32 * 32; }

// NB > 1 (the Q8-activation forms without the fused quantiser): a CTA takes
// NB activation rows (tokens) at once and streams the weights once for all
// of them; each token keeps its own dots and chains, so its result is the
// one-token result, bit for bit.
template <int MODE, bool FUSED, int R, int P, int CG, int NB = 1>
__global__ void __launch_bounds__(stream_consumers(R) + 32 * P, 2) k_q8_gemv_stream(GemvArgs p, int stages, int xstaged_arg)
{
	kernel_entry();
	static_assert(P >= 1 && P <= 4, "one to four producer warps");
	static_assert(NB == 1 || (MODE != 2 && !FUSED), "token blocks: the Q8-activation forms");
	constexpr int NM = MODE == 0 ? 1 : 2;
	constexpr int kConsumers = stream_consumers(R);
	static_assert(CG % 16 == 0, "whole 16-group batches per chunk");
	constexpr int kSlot = row_slot(CG);
	constexpr int kStageBytes = NM * R * kSlot;
	extern __shared__ __align__(128) unsigned char smem[];
	const int n = p.n, groups = n / kQ8Group;
	const int nchunks = (groups + CG - 1) / CG;
	const int64_t nrb = (p.d + R - 1) / R;
	const int64_t b = (int64_t)blockIdx.y * NB; // the block's first token
	const int nt = NB == 1 ? 1 : (int)min((int64_t)NB, (int64_t)p.batch - b);
	const int astride = n + 4 * (groups + 16); // bytes: a token's codes and scales
	// only the fp32-activation forms have a staging area in their layout
	const bool xstaged = (MODE == 2 || FUSED) && xstaged_arg != 0;
	const int mstride = R * groups; // floats between a slot's matrices
	float *sws = reinterpret_cast<float *>(smem + (size_t)stages * kStageBytes);
	unsigned char *act = reinterpret_cast<unsigned char *>(sws + 2 * NM * mstride + 16);
	uint32_t *sq = reinterpret_cast<uint32_t *>(act);
	float *ss = reinterpret_cast<float *>(act + n);
	float *xt = reinterpret_cast<float *>(act);
	const int xstride = groups * 8 + 4; // MODE 2: the 8 lanes' rows start 4 banks apart
	float *xstage = reinterpret_cast<float *>(reinterpret_cast<unsigned char *>(sws) + stream_fixed(MODE, R, n, NB));
	uint64_t *full = reinterpret_cast<uint64_t *>(reinterpret_cast<unsigned char *>(xstage) + (xstaged ? 4 * (size_t)n : 0));
	uint64_t *empty = full + stages;
	uint64_t *sfull = empty + stages;
	uint64_t *sempty = sfull + 2;
	uint64_t *pro = sempty + 2;
	if (threadIdx.x == 0) {
		for (int s = 0; s < stages; ++s) {
			mbar_init(full + s, P); // one arrival (with its byte count) per producer warp
			mbar_init(empty + s, kConsumers / 32);
		}
		for (int s = 0; s < 2; ++s) {
			mbar_init(sfull + s, 1);
			mbar_init(sempty + s, kConsumers / 32);
		}
		mbar_init(pro, 1);
		mbar_init_fence();
	}
	__syncthreads();
	const bool pro_copy = (MODE != 2 && !FUSED) || xstaged;
	// FUSED: the consumer warps quantise the activation while the producers
	// issue the first weight chunks, then meet at named barrier 2 (consumers
	// only).  With the producers taking part the barrier waited for them to
	// get their first stages issued, which the memory system paces: the
	// activation was quantised 1.9 us after its copy landed instead of by the
	// time the first chunk had (v7d_q8_fused 8192 -> 2048: 7.72 -> 7.21 us).
	// Each consumer thread arrives there exactly once and waits for nothing
	// unbounded before it.
	auto quantise_all = [&]() {
		if (xstaged) {
			mbar_wait(pro, 0, &g_pipeline_timeouts);
			stage_quantized<true, true>(xstage, n, sq, ss, kConsumers);
		} else {
			stage_quantized<false, true>(p.xf + b * n, n, sq, ss, kConsumers);
		}
		named_sync(2, kConsumers);
	};
	if (threadIdx.x >= kConsumers) {
		// P producer warps: warp 0 also copies the activation and the scales;
		// the copies of a stage are dealt round-robin (a warp issues one copy
		// per active lane, and issuing costs the warp tens of cycles per copy,
		// so one warp alone cannot keep HBM busy with 1 KB copies)
		const int lane = threadIdx.x & 31;
		const int pw = (threadIdx.x - kConsumers) >> 5;
		if (pro_copy && pw == 0 && lane == 0) {
			if (MODE != 2 && !FUSED) {
				mbar_arrive_expect_tx(pro, (uint32_t)(nt * (n + 4 * groups)));
				for (int t = 0; t < nt; ++t) {
					bulk_copy_g2s(act + t * astride, p.xq + (b + t) * n, (uint32_t)n, pro);
					bulk_copy_g2s(act + t * astride + n, p.xs + (b + t) * groups, (uint32_t)(4 * groups), pro);
				}
			} else {
				mbar_arrive_expect_tx(pro, (uint32_t)(4 * n));
				bulk_copy_g2s(xstage, p.xf + b * n, (uint32_t)(4 * n), pro);
			}
		}
		uint32_t q = 0;
		int i = 0;
		bool ok = true;
		for (int64_t rb = blockIdx.x; rb < nrb && ok; rb += gridDim.x, ++i) {
			const int64_t row0 = rb * R;
			const int rows = (int)min((int64_t)R, p.d - row0);
			const int slot = i & 1;
			if (pw == 0) {
				if (i >= 2 && lane == 0)
					ok = mbar_wait(sempty + slot, ((i >> 1) - 1) & 1, &g_pipeline_timeouts);
				if (!__shfl_sync(0xffffffffu, ok, 0))
					break;
				if (lane == 0)
					mbar_arrive_expect_tx(sfull + slot, (uint32_t)(NM * rows * groups * 4));
				__syncwarp();
				if (lane < NM)
					bulk_copy_g2s(sws + (slot * NM + lane) * mstride, (lane == 0 ? p.ws[0] : p.ws[NM - 1]) + row0 * groups,
					              (uint32_t)(rows * groups * 4), sfull + slot);
			}
			const int ncopy = NM * rows;
			const int mine = ncopy > pw ? (ncopy - pw + P - 1) / P : 0; // copies pw, pw + P, ...
			for (int k = 0; k < nchunks; ++k, ++q) {
				const int s = (int)(q % (uint32_t)stages);
				if (q >= (uint32_t)stages && lane == 0)
					ok = mbar_wait(empty + s, ((q / stages) - 1) & 1, &g_pipeline_timeouts);
				if (!__shfl_sync(0xffffffffu, ok, 0))
					break;
				const int g0 = k * CG;
				const int gk = min(CG, groups - g0);
				const uint32_t bytes = (uint32_t)(gk * kQ8Group);
				if (lane == 0)
					mbar_arrive_expect_tx(full + s, bytes * (uint32_t)mine);
				__syncwarp();
				if (lane < mine) {
					const int c = pw + P * lane;
					const int m = c / rows, r = c - m * rows;
					// a select, not p.wq[m]: a runtime index into the parameter
					// array would copy it to local memory
					const int8_t *wm = m == 0 ? p.wq[0] : p.wq[NM - 1];
					bulk_copy_g2s(smem + (size_t)s * kStageBytes + (m * R + r) * kSlot, wm + (row0 + r) * n + (int64_t)g0 * kQ8Group, bytes,
					              full + s);
				}
			}
		}
		// leave only once every copy issued has landed
		if (lane == 0) {
			for (uint32_t k = q > (uint32_t)stages ? q - stages : 0; k < q; ++k)
				if (!mbar_wait(full + k % stages, (k / stages) & 1, &g_pipeline_timeouts))
					break;
			if (pw == 0) {
				for (int j = i > 2 ? i - 2 : 0; j < i; ++j)
					if (!mbar_wait(sfull + (j & 1), (j >> 1) & 1, &g_pipeline_timeouts))
						break;
				if (pro_copy)
					mbar_wait(pro, 0, &g_pipeline_timeouts);
			}
		}
		return;
	}
	// consumers.  A wait that runs out clears the warp's `live` flag: the warp
	// skips its remaining waits and arithmetic but still reaches every named
	// barrier below, so the other warps' barriers complete; nothing is stored.
	bool live = !pro_copy || __all_sync(0xffffffffu, mbar_wait(pro, 0, &g_pipeline_timeouts));
	if (MODE == 2) {
		const float *xb = p.xf + b * n;
		for (int e = threadIdx.x; e < n; e += kConsumers)
			xt[(e & 7) * xstride + (e >> 6) * 8 + ((e >> 3) & 7)] = xstaged ? xstage[e] : __ldg(xb + e);
		named_sync(1, kConsumers);
	}
	if (FUSED)
		quantise_all();
	if (MODE != 2 && !FUSED) {
		// the copied codes into the interleaved layout, in place: word 2l of a
		// group = word l, word 2l + 1 = word 8 + l (one 8-byte load per lane and group)
		for (int t = 0; t < nt; ++t)
			for (int g = threadIdx.x; g < groups; g += kConsumers) {
				uint4 *pg = reinterpret_cast<uint4 *>(act + t * astride) + g * 4;
				const uint4 q0 = pg[0], q1 = pg[1], q2 = pg[2], q3 = pg[3];
				pg[0] = make_uint4(q0.x, q2.x, q0.y, q2.y);
				pg[1] = make_uint4(q0.z, q2.z, q0.w, q2.w);
				pg[2] = make_uint4(q1.x, q3.x, q1.y, q3.y);
				pg[3] = make_uint4(q1.z, q3.z, q1.w, q3.w);
			}
		named_sync(1, kConsumers);
	}
	const int r = threadIdx.x / kLanes, l = threadIdx.x & (kLanes - 1);
	uint32_t q = 0;
	int i = 0;
	for (int64_t rb = blockIdx.x; rb < nrb; rb += gridDim.x, ++i) {
		const int64_t row0 = rb * R;
		const int rows = (int)min((int64_t)R, p.d - row0);
		const bool valid = r < rows;
		const int slot = i & 1;
		live = live && __all_sync(0xffffffffu, mbar_wait(sfull + slot, (i >> 1) & 1, &g_pipeline_timeouts));
		// (the fused form keeps forming it per group: measured 7.19 -> 7.49 us
		// at d = 2048, n = 8192 with it, while v7d_q8 went 6.72 -> 6.59 us)
		constexpr bool kCombined = MODE == 0 && NB == 1 && !FUSED;
		if constexpr (kCombined) {
			// the warp's rows (at most four, within the slot's R): weight scale x
			// activation scale rounded once, as the reference's vmulps, in place --
			// once per row instead of once per lane thread and group
			using M = F<true>;
			const int w = threadIdx.x >> 5;
			const int wrows = min(4, R - 4 * w);
			float4 *sw4 = reinterpret_cast<float4 *>(sws + slot * mstride + 4 * w * groups);
			const float4 *ss4 = reinterpret_cast<const float4 *>(ss);
			for (int e = threadIdx.x & 31; e < wrows * groups / 4; e += 32) {
				float4 w4 = sw4[e];
				const float4 x4 = ss4[e % (groups / 4)];
				w4.x = M::mul(w4.x, x4.x), w4.y = M::mul(w4.y, x4.y), w4.z = M::mul(w4.z, x4.z), w4.w = M::mul(w4.w, x4.w);
				sw4[e] = w4;
			}
			__syncwarp();
		}
		const float *wsr = sws + slot * NM * mstride + r * groups;
		float acc[NM][NB];
#pragma unroll
		for (int m = 0; m < NM; ++m)
#pragma unroll
			for (int t = 0; t < NB; ++t)
				acc[m][t] = 0.0f;
		for (int k = 0; k < nchunks; ++k, ++q) {
			const int s = (int)(q % (uint32_t)stages);
			const int g0 = k * CG;
			const int gk = min(CG, groups - g0);
			// warp-uniform: the warp waits, and computes, together
			live = live && __all_sync(0xffffffffu, mbar_wait(full + s, (q / stages) & 1, &g_pipeline_timeouts));
			if (live && valid) {
				const uint32_t *st = reinterpret_cast<const uint32_t *>(smem + (size_t)s * kStageBytes) + r * (kSlot / 4);
				if constexpr (MODE == 2) {
					float a2[2] = {acc[0][0], acc[NM - 1][0]};
					chunk_f32<R, CG>(a2, st, xt + l * xstride + g0 * 8, wsr + g0, groups, l, gk);
					acc[0][0] = a2[0];
					acc[NM - 1][0] = a2[1];
				} else if constexpr (NM == 1) { // 16-group batches (8 for token blocks), the most independent work per wait
					constexpr int SB = NB == 1 ? 16 : 8;
					if constexpr (NB == 1) {
						if (gk == CG)
							chunk_chain1_one<R, 16, CG, true, kCombined>(acc[0][0], st, sq + g0 * 16, wsr + g0, ss + g0, l, CG);
						else
							chunk_chain1_one<R, 16, CG, false, kCombined>(acc[0][0], st, sq + g0 * 16, wsr + g0, ss + g0, l, gk);
					} else if (gk == CG) {
						chunk_chain1<NB, SB, CG, true>(acc[0], st, sq + g0 * 16, astride / 4, wsr + g0, ss + g0, astride / 4, l, CG);
					} else {
						chunk_chain1<NB, SB, CG, false>(acc[0], st, sq + g0 * 16, astride / 4, wsr + g0, ss + g0, astride / 4, l, gk);
					}
				} else {
					constexpr int SB = NB == 4 ? 4 : 8;
					if (gk == CG) // a constant bound: no group needs a check
						chunk_chains_ws<NM, NB, R, SB, CG>(acc, st, sq + g0 * 16, astride / 4, wsr + g0, mstride, ss + g0, astride / 4, l, CG);
					else
						chunk_chains_ws<NM, NB, R, SB, CG>(acc, st, sq + g0 * 16, astride / 4, wsr + g0, mstride, ss + g0, astride / 4, l, gk);
				}
			}
			__syncwarp();
			if ((threadIdx.x & 31) == 0)
				mbar_arrive(empty + s);
		}
#pragma unroll
		for (int t = 0; t < NB; ++t) {
			float res[NM];
#pragma unroll
			for (int m = 0; m < NM; ++m)
				res[m] = hadd_lanes(acc[m][t]);
			if (live && valid && l == 0 && t < nt)
				p.out[(b + t) * p.d + row0 + r] = MODE == 0 ? res[0] : v7_swiglu(res[0], res[NM - 1]);
		}
		if constexpr (kCombined)
			fence_proxy_async_smem(); // the slot's next fill is a bulk copy over these writes
		__syncwarp();
		if ((threadIdx.x & 31) == 0)
			mbar_arrive(sempty + slot);
	}
}

// Shared memory of k_q8_gemv_tma for `stages` stages.
size_t tma_smem(int mode, int rows, int n, int stages)
{
	const int nm = mode == 0 ? 1 : 2;
	const int groups = n / kQ8Group;
	const size_t act = mode == 2 ? 32 * ((size_t)groups * 8 + 4) : (size_t)n + 4 * (size_t)groups;
	const size_t fixed = act + 4 * (size_t)nm * rows * (groups + 1) + 8 + 16 * (size_t)stages;
	return (size_t)stages * nm * rows * kRowSlot + fixed;
}

// fp32 activation x Q8 weights, SwiGLU epilogue (v7d_swiglu, dual-row path):
// thread l of a row owns lane l, i.e. elements e = l (mod 8).
__global__ void __launch_bounds__(kBlock) k_f32q8_swiglu_gemv(GemvArgs p)
{
	kernel_entry();
	using M = F<true>;
	const int n = p.n, groups = n / kQ8Group;
	const int64_t b = blockIdx.y;
	const int l = threadIdx.x & (kLanes - 1);
	const int64_t row_raw = (int64_t)blockIdx.x * kRowsPerBlock + (threadIdx.x >> 3);
	const bool valid = row_raw < p.d;
	const int64_t row = valid ? row_raw : 0;
	const int gend = valid ? groups : 0;
	const float *x = p.xf + b * n + l;
	const int8_t *w[2] = {p.wq[0] + row * n + l, p.wq[1] + row * n + l};
	const float *s[2] = {p.ws[0] + row * groups, p.ws[1] + row * groups};
	float acc[2] = {0.0f, 0.0f};
	for (int g = 0; g < gend; ++g) {
		int8_t wb[2][8];
		float xv[8];
#pragma unroll
		for (int k = 0; k < 8; ++k) {
			wb[0][k] = __ldcs(w[0] + g * kQ8Group + 8 * k);
			wb[1][k] = __ldcs(w[1] + g * kQ8Group + 8 * k);
			xv[k] = __ldg(x + g * kQ8Group + 8 * k);
		}
		const float sg[2] = {__ldg(s[0] + g), __ldg(s[1] + g)};
#pragma unroll
		for (int k = 0; k < 8; ++k)
#pragma unroll
			for (int m = 0; m < 2; ++m)
				acc[m] = M::fma(xv[k], M::mul((float)wb[m][k], sg[m]), acc[m]);
	}
	const float gsum = hadd_lanes(acc[0]), usum = hadd_lanes(acc[1]);
	if (l == 0 && valid)
		p.out[b * p.d + row] = v7_swiglu(gsum, usum);
}

int check_gemv(const char *what, float *out, int64_t batch, int n, int d)
{
	if (batch < 0 || d < 0)
		return set_error(V7G_ERR_ARG, "%s: negative batch or d", what);
	if (n <= 0 || n % kQ8Group != 0 || n > kMaxN)
		return set_error(V7G_ERR_ARG, "%s: n = %d must be a positive multiple of 64, at most %d", what, n, kMaxN);
	if (batch > 65535)
		return set_error(V7G_ERR_ARG, "%s: batch %lld above 65535", what, (long long)batch);
	if (batch > 0 && d > 0 && !out)
		return set_error(V7G_ERR_ARG, "%s: NULL output", what);
	return V7G_OK;
}

template <typename Kernel>
int launch_gemv(Kernel kernel, const char *what, const GemvArgs &a, int64_t batch, size_t smem, void *stream)
{
	DeviceInfo dev;
	int rc = current_device(&dev);
	if (rc != V7G_OK)
		return rc;
	if (smem > 48 * 1024 && cudaFuncSetAttribute((const void *)kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
		return check_launch(what);
	const dim3 grid((unsigned)((a.d + kRowsPerBlock - 1) / kRowsPerBlock), (unsigned)batch);
	const cudaError_t launched = launch_kernel(kernel, grid, kBlock, smem, stream, a);
	return check_launch(what, launched);
}

bool weights_ok(const int8_t *q, const float *s) { return q && s && (reinterpret_cast<uintptr_t>(q) & 3) == 0; }

constexpr size_t kTmaSmemBudget = 200 * 1024;
constexpr int kMaxDevicesTracked = 64;

// The pipelined kernel: R = 16 rows per CTA when that still gives two CTAs
// per SM, else 8; as many stages (up to 6) as the shared-memory budget
// allows.  Returns V7G_ERR_UNSUPPORTED when even two stages do not fit (a
// very long activation row), for the caller to fall back.
template <int MODE, bool FUSED>
int launch_gemv_tma(const char *what, const GemvArgs &a, int64_t batch, void *stream)
{
	DeviceInfo dev;
	int rc = current_device(&dev);
	if (rc != V7G_OK)
		return rc;
	const bool wide = a.d >= 2 * 16 * (int64_t)dev.sm_count;
	const int R = wide ? 16 : 8;
	// up to 4 stages while a CTA stays under ~112 KB (two per SM), at least 2
	int stages = 4;
	while (stages > 2 && tma_smem(MODE, R, a.n, stages) > 112 * 1024)
		--stages;
	while (stages > 2 && tma_smem(MODE, R, a.n, stages) > kTmaSmemBudget)
		--stages;
	const size_t smem = tma_smem(MODE, R, a.n, stages);
	if (smem > kTmaSmemBudget)
		return V7G_ERR_UNSUPPORTED;
	const void *kernel = wide ? (const void *)k_q8_gemv_tma<MODE, FUSED, 16> : (const void *)k_q8_gemv_tma<MODE, FUSED, 8>;
	// the shared-memory ceiling of each kernel is raised once per device (the
	// call is idempotent, so threads racing to the first launch may both make it)
	static std::atomic<bool> raised[2][kMaxDevicesTracked];
	if (dev.device < kMaxDevicesTracked && !raised[wide][dev.device].load(std::memory_order_relaxed)) {
		if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTmaSmemBudget) != cudaSuccess)
			return check_launch(what);
		raised[wide][dev.device].store(true, std::memory_order_relaxed);
	} else if (dev.device >= kMaxDevicesTracked &&
	           cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTmaSmemBudget) != cudaSuccess) {
		return check_launch(what);
	}
	const dim3 grid((unsigned)((a.d + R - 1) / R), (unsigned)batch);
	cudaError_t launched;
	if (wide)
		launched = launch_kernel((k_q8_gemv_tma<MODE, FUSED, 16>), grid, 16 * kLanes + 32, smem, stream, a, stages);
	else
		launched = launch_kernel((k_q8_gemv_tma<MODE, FUSED, 8>), grid, 8 * kLanes + 32, smem, stream, a, stages);
	return check_launch(what, launched);
}

// Per-CTA shared memory aimed at two CTAs per SM, or one when two stages do
// not fit that way or when there are no more row blocks than SMs (one CTA
// per SM then in any case, so it may as well take the whole SM).
constexpr size_t kStreamSmemTwo = 110 * 1024;
constexpr size_t kStreamSmemOne = 220 * 1024;

StreamLayout stream_layout(int mode, bool fused, int rows_per_block, int n, bool x_aligned, int cg, bool one_per_sm = false, int tokens = 1)
{
	const int nm = mode == 0 ? 1 : 2;
	const size_t stage = (size_t)nm * rows_per_block * row_slot(cg);
	const size_t bars = 8 * (2 * (size_t)kMaxStages + 5);
	const size_t fixed = stream_fixed(mode, rows_per_block, n, tokens) + bars;
	const bool want_x = (mode == 2 || fused) && x_aligned;
	for (size_t budget : {one_per_sm ? kStreamSmemOne : kStreamSmemTwo, kStreamSmemOne})
		for (int xs = want_x ? 1 : 0; xs >= 0; --xs) {
			const size_t base = fixed + (xs ? 4 * (size_t)n : 0);
			if (base + 2 * stage > budget)
				continue;
			const int stages = (int)std::min<size_t>(mode == 0 ? (fused ? kMaxStagesFused : kMaxStagesOne) : kMaxStages, (budget - base) / stage);
			return StreamLayout{stages, xs != 0, base + (size_t)stages * stage};
		}
	return StreamLayout{0, false, 0};
}

// Streaming-kernel shapes, measured on B200 at the decode shapes (d = 2048
// .. 12288): 2 KB row copies for the one-matrix product, 1 KB for the
// two-matrix ones (their stages are twice as big); two producer warps (four
// measured slower for v7d_q8 at d = 2048, n = 8192: 6.80 against 6.72 us).
// Rows per block: 16, or 14 where that spreads the row blocks more evenly
// over the SMs (launch_gemv_stream); fewer rows per block than that keep too
// few bytes in flight per CTA.
template <int MODE, bool FUSED>
struct StreamShape {
	static constexpr int P = 2;
	static constexpr int CG = MODE == 0 ? 32 : kChunkGroups;
};

// The most rows any SM streams when `nrb` row blocks of R rows are walked by
// `grid` CTAs (CTA c takes blocks c, c + grid, ...; CTA c sits on SM
// c % sm_count).
int64_t busiest_sm_rows(int64_t nrb, int64_t grid, int sm_count, int rows_per_block)
{
	int64_t worst = 0;
	for (int64_t sm = 0; sm < std::min<int64_t>(grid, sm_count); ++sm) {
		int64_t blocks = 0;
		for (int64_t c = sm; c < grid; c += sm_count)
			blocks += (nrb - c + grid - 1) / grid;
		worst = std::max(worst, blocks);
	}
	return worst * rows_per_block;
}

struct StreamPlan {
	StreamLayout lay;
	const void *kernel;
	int threads;
	dim3 grid;
	int64_t busiest;
};

// The layout, kernel and grid of one rows-per-block choice with NB tokens a
// CTA; busiest < 0 when it does not fit (or groups % 4 != 0).
template <int MODE, bool FUSED, int R, int NB>
int plan_stream(const char *what, const GemvArgs &a, int64_t batch, const DeviceInfo &dev, StreamPlan &plan)
{
	using S = StreamShape<MODE, FUSED>;
	plan.busiest = -1;
	const int64_t nrb = (a.d + R - 1) / R;
	const int64_t blocks_y = (batch + NB - 1) / NB;
	plan.lay = stream_layout(MODE, FUSED, R, a.n, aligned16(a.xf), S::CG, nrb * blocks_y <= dev.sm_count, NB);
	if (plan.lay.stages < 2)
		return V7G_OK;
	plan.kernel = (const void *)k_q8_gemv_stream<MODE, FUSED, R, S::P, S::CG, NB>;
	plan.threads = stream_consumers(R) + 32 * S::P;
	// the shared-memory ceiling of the kernel is raised once per device
	static std::atomic<bool> raised[kMaxDevicesTracked];
	if (dev.device >= kMaxDevicesTracked || !raised[dev.device].load(std::memory_order_relaxed)) {
		if (cudaFuncSetAttribute(plan.kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kStreamSmemOne) != cudaSuccess)
			return check_launch(what);
		if (dev.device < kMaxDevicesTracked)
			raised[dev.device].store(true, std::memory_order_relaxed);
	}
	int per_sm = 0;
	if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, plan.kernel, plan.threads, plan.lay.smem) != cudaSuccess || per_sm < 1)
		return check_launch(what);
	const int64_t slots = std::max<int64_t>(1, (int64_t)per_sm * dev.sm_count / blocks_y);
	plan.grid = dim3((unsigned)std::min(nrb, slots), (unsigned)blocks_y);
	plan.busiest = busiest_sm_rows(nrb, plan.grid.x, dev.sm_count, R);
	return V7G_OK;
}

// grid = the resident CTAs (split over the token blocks), at most one per
// row block; 16 or 14 rows per block, whichever leaves the busiest SM fewer
// rows (16 on a tie).  V7G_ERR_UNSUPPORTED when the layout does not fit, for
// the caller to fall back.
template <int MODE, bool FUSED, int NB>
int launch_stream_tokens(const char *what, const GemvArgs &a, int64_t batch, const DeviceInfo &dev, void *stream)
{
	using S = StreamShape<MODE, FUSED>;
	StreamPlan p16, p14;
	int rc;
	if ((rc = plan_stream<MODE, FUSED, 16, NB>(what, a, batch, dev, p16)) != V7G_OK || (rc = plan_stream<MODE, FUSED, 14, NB>(what, a, batch, dev, p14)) != V7G_OK)
		return rc;
	const bool use14 = p14.busiest >= 0 && (p16.busiest < 0 || p14.busiest < p16.busiest);
	const StreamPlan &pl = use14 ? p14 : p16;
	if (pl.busiest < 0)
		return V7G_ERR_UNSUPPORTED;
	const int stages = pl.lay.stages, xs = pl.lay.xstaged ? 1 : 0;
	const cudaError_t launched =
	    use14 ? launch_kernel((k_q8_gemv_stream<MODE, FUSED, 14, S::P, S::CG, NB>), pl.grid, pl.threads, pl.lay.smem, stream, a, stages, xs)
	          : launch_kernel((k_q8_gemv_stream<MODE, FUSED, 16, S::P, S::CG, NB>), pl.grid, pl.threads, pl.lay.smem, stream, a, stages, xs);
	return check_launch(what, launched);
}

// The Q8-activation forms without the fused quantiser take 2 tokens a CTA
// for a batch of 2 and 4 from 3 on, so the weights stream once per four
// activation rows instead of once per row; groups % 4 != 0 is unsupported.
template <int MODE, bool FUSED>
int launch_gemv_stream(const char *what, const GemvArgs &a, int64_t batch, void *stream)
{
	if ((a.n / kQ8Group) % 4 != 0)
		return V7G_ERR_UNSUPPORTED;
	DeviceInfo dev;
	int rc = current_device(&dev);
	if (rc != V7G_OK)
		return rc;
	// a block whose activations do not fit beside two stages (long rows)
	// steps down to fewer tokens a CTA
	if constexpr (MODE != 2 && !FUSED) {
		if (batch >= 3 && (rc = launch_stream_tokens<MODE, FUSED, 4>(what, a, batch, dev, stream)) != V7G_ERR_UNSUPPORTED)
			return rc;
		if (batch >= 2 && (rc = launch_stream_tokens<MODE, FUSED, 2>(what, a, batch, dev, stream)) != V7G_ERR_UNSUPPORTED)
			return rc;
	}
	return launch_stream_tokens<MODE, FUSED, 1>(what, a, batch, dev, stream);
}

// The streaming kernel when weights and scales allow bulk copies (16-byte
// aligned), else the pipelined kernel when the weights do, else (or when
// neither fits) the direct-load kernel.
template <int MODE, bool FUSED>
int run_q8_gemv(const char *what, const GemvArgs &a, int64_t batch, void *stream, bool tma, bool scales16)
{
	if (tma && scales16) {
		const int rc = launch_gemv_stream<MODE, FUSED>(what, a, batch, stream);
		if (rc != V7G_ERR_UNSUPPORTED)
			return rc;
	}
	if (tma) {
		const int rc = launch_gemv_tma<MODE, FUSED>(what, a, batch, stream);
		if (rc != V7G_ERR_UNSUPPORTED)
			return rc;
	}
	return launch_gemv(k_q8_gemv<MODE, FUSED>, what, a, batch, (size_t)a.n + (size_t)a.n / 16, stream);
}

} // namespace
} // namespace v7g

using namespace v7g;

extern "C" {

int v7g_q8_gemv(float *out, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws, int64_t batch, int n, int d, void *stream)
{
	const char *what = "v7g_q8_gemv";
	int rc = check_gemv(what, out, batch, n, d);
	if (rc != V7G_OK)
		return rc;
	if (batch == 0 || d == 0)
		return clear_error();
	if (!xq || !xs || !aligned16(xq) || !weights_ok(wq, ws))
		return set_error(V7G_ERR_ARG, "%s: NULL pointer, activation codes not 16-byte or weight codes not 4-byte aligned", what);
	GemvArgs a{out, xq, xs, nullptr, {wq, wq}, {ws, ws}, n, d, (int)batch};
	return run_q8_gemv<0, false>(what, a, batch, stream, aligned16(wq), aligned16(ws) && aligned16(xs));
}

int v7g_q8_fused_gemv(float *out, const float *x, const int8_t *wq, const float *ws, int64_t batch, int n, int d, void *stream)
{
	const char *what = "v7g_q8_fused_gemv";
	int rc = check_gemv(what, out, batch, n, d);
	if (rc != V7G_OK)
		return rc;
	if (batch == 0 || d == 0)
		return clear_error();
	if (!x || !weights_ok(wq, ws))
		return set_error(V7G_ERR_ARG, "%s: NULL pointer or weight codes not 4-byte aligned", what);
	GemvArgs a{out, nullptr, nullptr, x, {wq, wq}, {ws, ws}, n, d, (int)batch};
	return run_q8_gemv<0, true>(what, a, batch, stream, aligned16(wq), aligned16(ws));
}

int v7g_swiglu_q8_gemv(float *out, const int8_t *xq, const float *xs, const int8_t *gate_q, const float *gate_s, const int8_t *up_q, const float *up_s, int64_t batch, int n, int d, void *stream)
{
	const char *what = "v7g_swiglu_q8_gemv";
	int rc = check_gemv(what, out, batch, n, d);
	if (rc != V7G_OK)
		return rc;
	if (batch == 0 || d == 0)
		return clear_error();
	if (!xq || !xs || !aligned16(xq) || !weights_ok(gate_q, gate_s) || !weights_ok(up_q, up_s))
		return set_error(V7G_ERR_ARG, "%s: NULL pointer, activation codes not 16-byte or weight codes not 4-byte aligned", what);
	GemvArgs a{out, xq, xs, nullptr, {gate_q, up_q}, {gate_s, up_s}, n, d, (int)batch};
	return run_q8_gemv<1, false>(what, a, batch, stream, aligned16(gate_q) && aligned16(up_q),
	                             aligned16(gate_s) && aligned16(up_s) && aligned16(xs));
}

int v7g_swiglu_f32q8_gemv(float *out, const float *x, const int8_t *gate_q, const float *gate_s, const int8_t *up_q, const float *up_s, int64_t batch, int n, int d, void *stream)
{
	const char *what = "v7g_swiglu_f32q8_gemv";
	int rc = check_gemv(what, out, batch, n, d);
	if (rc != V7G_OK)
		return rc;
	if (batch == 0 || d == 0)
		return clear_error();
	if (!x || !gate_q || !gate_s || !up_q || !up_s)
		return set_error(V7G_ERR_ARG, "%s: NULL pointer", what);
	GemvArgs a{out, nullptr, nullptr, x, {gate_q, up_q}, {gate_s, up_s}, n, d, (int)batch};
	if (aligned16(gate_q) && aligned16(up_q) && aligned16(gate_s) && aligned16(up_s)) {
		const int rc2 = launch_gemv_stream<2, false>(what, a, batch, stream);
		if (rc2 != V7G_ERR_UNSUPPORTED)
			return rc2;
	}
	if (aligned16(gate_q) && aligned16(up_q)) {
		const int rc2 = launch_gemv_tma<2, false>(what, a, batch, stream);
		if (rc2 != V7G_ERR_UNSUPPORTED)
			return rc2;
	}
	return launch_gemv(k_f32q8_swiglu_gemv, what, a, batch, 0, stream);
}

unsigned int v7g_pipeline_timeouts(void)
{
	unsigned int v = 0;
	if (cudaMemcpyFromSymbol(&v, g_pipeline_timeouts, sizeof(v)) != cudaSuccess) {
		cudaGetLastError();
		return 0xffffffffu;
	}
	const unsigned int a = v7g::norm_pipe_timeouts(), b = v7g::norm_q8_pipe_timeouts();
	if (a == 0xffffffffu || b == 0xffffffffu)
		return 0xffffffffu;
	return v + a + b;
}

} // extern "C"
