// rope.cu -- per-head RMSNorm + NeoX half-split RoPE over GQA Q/K, in place.
//
// Work item = (token, tensor Q or K, chunk of up to kChunk heads); one warp
// per item.  A head of D = 32*V floats is V slots per lane (element l + 32k),
// which is exactly the reference's sum-of-squares chain layout
// (RMSNORM_ROPE_BODY, v7_macros.inc:266-289).  For even V the rotation
// partners j and j + D/2 are slots k and k + V/2 of the same lane, so the head
// never leaves registers; the token's cos/sin row and both gamma vectors are
// loaded once per item / once per warp.  Other head sizes take a general
// kernel that re-reads the head (from L1) in the rotation pass.
// The reference runs this kernel on its dispatched workers: FTZ+DAZ.
#include "internal.h"
#include "launch.cuh"
#include "reduce.cuh"

namespace v7g {
namespace {

constexpr int kBlock = 256;
// heads per warp work item
constexpr int kChunk = 4;

// 1/sqrt(ss / D + eps) in v7's order (COMPUTE_RMS_SCALE, v7_macros.inc:348-354)
// with cheaper exact steps: for a power-of-two D, ss / D is the exact product
// ss * (1/D) (FTZ flushes a subnormal quotient either way), and the final
// reciprocal takes the Markstein form (exact for normal arguments with normal
// reciprocals; zero, subnormal, inf and NaN take rcp.rn).
template <int D>
__device__ __forceinline__ float head_rms_scale(float ss, float eps)
{
	using M = F<true>;
	constexpr bool pow2 = (D & (D - 1)) == 0;
	const float mean = pow2 ? M::mul(ss, 1.0f / (float)D) : M::div(ss, (float)D);
	const float r = M::sqrt(M::add(mean, eps));
	return (r >= 1.17549435e-38f && r < 8.50705917e37f) ? rcp_nr_ftz(r) : M::rcp(r);
}

// reduce_chains_4x8 of four heads at once.  The butterfly pairs lanes at
// distance 8, 16, 4, 1, 2 as reduce_chains_4x8 does, but after the first
// step a lane keeps the partial sums of only two heads (bit 3 of the lane
// picks which two) and after the second of one (bit 4), so one shuffle moves
// what the partner needs instead of four.  Each head's total is the same
// pairwise tree of the same values as reduce_chains_4x8 gives (fp32 addition
// is commutative), so it is bit-identical; head h's total lands in the lanes
// with bit 3 = h >> 1 and bit 4 = h & 1.
__device__ __forceinline__ float reduce_chains_4x8_quad(const float (&a)[4], int lane)
{
	using M = F<true>;
	const bool b3 = (lane & 8) != 0, b4 = (lane & 16) != 0;
	// distance 8: keep heads {0, 1} (bit 3 clear) or {2, 3}, send the other pair
	const float r0 = __shfl_xor_sync(kFullMask, b3 ? a[0] : a[2], 8);
	const float r1 = __shfl_xor_sync(kFullMask, b3 ? a[1] : a[3], 8);
	const float s0 = M::add(b3 ? a[2] : a[0], r0);
	const float s1 = M::add(b3 ? a[3] : a[1], r1);
	// distance 16: keep the first (bit 4 clear) or the second of the pair
	const float r = __shfl_xor_sync(kFullMask, b4 ? s0 : s1, 16);
	float t = M::add(b4 ? s1 : s0, r);
	t = M::add(t, __shfl_xor_sync(kFullMask, t, 4));
	t = M::add(t, __shfl_xor_sync(kFullMask, t, 1));
	return M::add(t, __shfl_xor_sync(kFullMask, t, 2));
}

struct RopeArgs {
	float *q;
	float *k;
	const float *wq;
	const float *wk;
	const float *cos_t;
	const float *sin_t;
	int64_t tokens;
	int64_t pos0;
	int hq, hk;
	int rope_max_dim;
	float eps;
};

template <int V, int CH = kChunk>
__global__ void __launch_bounds__(kBlock) k_rope_rows(RopeArgs p)
{
	kernel_entry();
	using M = F<true>;
	constexpr int D = 32 * V;
	constexpr int P = V / 2;
	const int lane = threadIdx.x & 31;
	const int64_t nwarps = ((int64_t)gridDim.x * kBlock) >> 5;
	const int cq = (p.hq + CH - 1) / CH;
	const int ck = (p.hk + CH - 1) / CH;
	const int per_token = cq + ck;
	const int64_t total = p.tokens * per_token;
	float gq[V], gk[V];
#pragma unroll
	for (int k = 0; k < V; ++k) {
		gq[k] = p.hq ? __ldg(p.wq + lane + 32 * k) : 0.0f;
		gk[k] = p.hk ? __ldg(p.wk + lane + 32 * k) : 0.0f;
	}
	for (int64_t item = ((int64_t)blockIdx.x * kBlock + threadIdx.x) >> 5; item < total; item += nwarps) {
		const int64_t t = item / per_token;
		const int s = (int)(item - t * per_token);
		const bool isq = s < cq;
		const int heads = isq ? p.hq : p.hk;
		const int h0 = (isq ? s : s - cq) * CH;
		const int nh = min(CH, heads - h0);
		float *base = (isq ? p.q : p.k) + (t * heads + h0) * (int64_t)D + lane;
		const int64_t pos = p.pos0 + t;
		float c[P], sn[P];
		if (pos != 0) {
			const float *cr = p.cos_t + pos * p.rope_max_dim + lane;
			const float *sr = p.sin_t + pos * p.rope_max_dim + lane;
#pragma unroll
			for (int j = 0; j < P; ++j) {
				c[j] = __ldg(cr + 32 * j);
				sn[j] = __ldg(sr + 32 * j);
			}
		}
		float x[CH][V];
#pragma unroll
		for (int h = 0; h < CH; ++h)
			if (h < nh) {
#pragma unroll
				for (int k = 0; k < V; ++k)
					x[h][k] = ld_stream(base + h * D + 32 * k);
			}
		// per-head scales: four full heads share one butterfly and one scale
		// computation per lane (the lanes of class h hold head h's), else
		// one butterfly per head
		float hs[CH];
		if (CH == 4 && nh == 4) {
			float acc[4];
#pragma unroll
			for (int h = 0; h < 4; ++h) {
				acc[h] = 0.0f;
#pragma unroll
				for (int k = 0; k < V; ++k)
					acc[h] = M::fma(x[h][k], x[h][k], acc[h]);
			}
			const float mine = head_rms_scale<D>(reduce_chains_4x8_quad(acc, lane), p.eps);
#pragma unroll
			for (int h = 0; h < 4; ++h) // head h's lanes: 8 * (h >> 1) + 16 * (h & 1)
				hs[h] = __shfl_sync(kFullMask, mine, ((h >> 1) << 3) | ((h & 1) << 4));
		} else {
#pragma unroll
			for (int h = 0; h < CH; ++h)
				if (h < nh) {
					float acc = 0.0f;
#pragma unroll
					for (int k = 0; k < V; ++k)
						acc = M::fma(x[h][k], x[h][k], acc);
					hs[h] = head_rms_scale<D>(reduce_chains_4x8<true>(acc), p.eps);
				}
		}
#pragma unroll
		for (int h = 0; h < CH; ++h)
			if (h < nh) {
				const float scale = hs[h];
				float *hb = base + h * D;
				if (pos == 0) {
#pragma unroll
					for (int k = 0; k < V; ++k)
						st_stream(hb + 32 * k, M::mul(M::mul(x[h][k], scale), isq ? gq[k] : gk[k]));
				} else {
#pragma unroll
					for (int j = 0; j < P; ++j) {
						const float e = M::mul(M::mul(x[h][j], scale), isq ? gq[j] : gk[j]);
						const float o = M::mul(M::mul(x[h][j + P], scale), isq ? gq[j + P] : gk[j + P]);
						st_stream(hb + 32 * j, M::fma(-o, sn[j], M::mul(e, c[j])));
						st_stream(hb + 32 * (j + P), M::fma(o, c[j], M::mul(e, sn[j])));
					}
				}
			}
	}
}

// General head size (D % 32 == 0, D <= 1024): one warp per (token, head).
__global__ void __launch_bounds__(kBlock) k_rope_rows_general(RopeArgs p, int D)
{
	kernel_entry();
	using M = F<true>;
	const int lane = threadIdx.x & 31;
	const int64_t nwarps = ((int64_t)gridDim.x * kBlock) >> 5;
	const int V = D >> 5;
	const int half = D >> 1;
	const int per_token = p.hq + p.hk;
	const int64_t total = p.tokens * per_token;
	const float nf = (float)D;
	for (int64_t item = ((int64_t)blockIdx.x * kBlock + threadIdx.x) >> 5; item < total; item += nwarps) {
		const int64_t t = item / per_token;
		const int s = (int)(item - t * per_token);
		const bool isq = s < p.hq;
		const int heads = isq ? p.hq : p.hk;
		const int h = isq ? s : s - p.hq;
		float *hb = (isq ? p.q : p.k) + (t * heads + h) * (int64_t)D;
		const float *w = isq ? p.wq : p.wk;
		const int64_t pos = p.pos0 + t;
		float acc = 0.0f;
		for (int k = 0; k < V; ++k) {
			const float v = hb[lane + 32 * k];
			acc = M::fma(v, v, acc);
		}
		const float scale = rms_scale<true>(reduce_chains_4x8<true>(acc), nf, p.eps);
		__syncwarp();
		if (pos == 0) {
			for (int k = 0; k < V; ++k)
				hb[lane + 32 * k] = M::mul(M::mul(hb[lane + 32 * k], scale), __ldg(w + lane + 32 * k));
		} else {
			const float *cr = p.cos_t + pos * p.rope_max_dim;
			const float *sr = p.sin_t + pos * p.rope_max_dim;
			for (int j = lane; j < half; j += 32) {
				const float e = M::mul(M::mul(hb[j], scale), __ldg(w + j));
				const float o = M::mul(M::mul(hb[j + half], scale), __ldg(w + j + half));
				hb[j] = M::fma(-o, __ldg(sr + j), M::mul(e, __ldg(cr + j)));
				hb[j + half] = M::fma(o, __ldg(cr + j), M::mul(e, __ldg(sr + j)));
			}
		}
		__syncwarp();
	}
}

// Up to 4 x the blocks resident at once (at most work_blocks): a few waves of
// CTAs stream faster on B200 than exactly one resident wave.
template <typename Kernel, typename... Args>
int launch_persistent(Kernel kernel, const char *what, int64_t work_blocks, void *stream, Args... args)
{
	DeviceInfo dev;
	int rc = current_device(&dev);
	if (rc != V7G_OK)
		return rc;
	const int resident = resident_grid((const void *)kernel, kBlock, 0, work_blocks, dev);
	const int grid = (int)(work_blocks < 4ll * resident ? work_blocks : 4ll * resident);
	const cudaError_t launched = launch_kernel(kernel, grid, kBlock, 0, stream, args...);
	return check_launch(what, launched);
}

} // namespace
} // namespace v7g

using namespace v7g;

extern "C" int v7g_rmsnorm_rope_rows(float *q, float *k, int64_t tokens, int n_q_heads, int n_kv_heads, int head_dim, const float *wq, const float *wk, const float *cos_table, const float *sin_table, int64_t pos0, int rope_max_dim, float eps, void *stream)
{
	const char *what = "v7g_rmsnorm_rope_rows";
	if (head_dim < 32 || head_dim > 1024 || head_dim % 32 != 0)
		return set_error(V7G_ERR_ARG, "%s: head_dim = %d must be a multiple of 32 in [32, 1024]", what, head_dim);
	if (tokens < 0 || n_q_heads < 0 || n_kv_heads < 0 || pos0 < 0 || rope_max_dim < 0)
		return set_error(V7G_ERR_ARG, "%s: negative tokens, head count, pos0 or rope_max_dim", what);
	if ((n_q_heads > 0 && (!q || !wq)) || (n_kv_heads > 0 && (!k || !wk)))
		return set_error(V7G_ERR_ARG, "%s: NULL tensor or gamma for a non-empty head set", what);
	const bool rotates = tokens > 1 || pos0 > 0;
	if (rotates && (!cos_table || !sin_table))
		return set_error(V7G_ERR_ARG, "%s: NULL cos/sin table", what);
	if (tokens == 0 || n_q_heads + n_kv_heads == 0)
		return clear_error();
	RopeArgs a{q, k, wq, wk, cos_table, sin_table, tokens, pos0, n_q_heads, n_kv_heads, rope_max_dim, eps};
	const int V = head_dim / 32;
	const int per_token_chunks = (n_q_heads + kChunk - 1) / kChunk + (n_kv_heads + kChunk - 1) / kChunk;
	const int64_t chunk_blocks = (tokens * per_token_chunks + kBlock / 32 - 1) / (kBlock / 32);
	switch (V) {
	case 2:
		return launch_persistent(k_rope_rows<2>, what, chunk_blocks, stream, a);
	case 4:
		return launch_persistent(k_rope_rows<4>, what, chunk_blocks, stream, a);
	case 6:
		return launch_persistent(k_rope_rows<6>, what, chunk_blocks, stream, a);
	case 8:
		return launch_persistent(k_rope_rows<8>, what, chunk_blocks, stream, a);
	default: {
		const int64_t blocks = (tokens * (n_q_heads + n_kv_heads) + kBlock / 32 - 1) / (kBlock / 32);
		return launch_persistent(k_rope_rows_general, what, blocks, stream, a, head_dim);
	}
	}
}
