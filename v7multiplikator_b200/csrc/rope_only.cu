// rope_only.cu -- NeoX half-split RoPE without the norm over GQA Q/K, in place
// (v7s_rope_only_heads, rope_only_kernel.inc:11-53, rope_only_dispatch.inc:10-47:
// the path of models without a QK norm, forward_q8.inc:40-44).
//
// Per head of D floats and half = D/2: at position 0 nothing is written (the
// reference skips the head, cos = 1, sin = 0); otherwise every pair (lo, hi) =
// (x[j], x[j + half]) becomes
//     x[j]        = fma(-hi, sin_j, lo * cos_j)
//     x[j + half] = fma( hi, cos_j, lo * sin_j)
// with lo * cos_j and lo * sin_j rounded first (vmulps) and the hi term fused
// (vfnmadd231ps / vfmadd231ps, rope_only_kernel.inc:32-35).  The reference
// runs it on its dispatched workers with FTZ+DAZ (rope_only_dispatch.inc:30).
//
// No reduction couples the pairs, so the kernel is a flat stream: work item =
// four consecutive pairs of one head (float4 of lo, of hi, of cos, of sin);
// the token's cos/sin row is shared by all its heads and stays in L1/L2.
#include "internal.h"
#include "launch.cuh"
#include "reduce.cuh"

namespace v7g {
namespace {

constexpr int kBlock = 256;

struct RopeOnlyArgs {
	float *q;
	float *k;
	const float *cos_t;
	const float *sin_t;
	int64_t tokens;
	int64_t pos0;
	int hq, hk;
	int half;
	int rope_max_dim;
};

__device__ __forceinline__ void rotate(float lo, float hi, float c, float s, float &out_lo, float &out_hi)
{
	using M = F<true>;
	out_lo = M::fma(-hi, s, M::mul(lo, c));
	out_hi = M::fma(hi, c, M::mul(lo, s));
}

// VEC: every pointer 16-byte aligned and rope_max_dim % 4 == 0; an item is 4
// pairs.  Otherwise an item is one pair.
template <bool VEC>
__global__ void __launch_bounds__(kBlock) k_rope_only_rows(RopeOnlyArgs p)
{
	kernel_entry();
	constexpr int P = VEC ? 4 : 1;
	const int per_head = p.half / P;
	const int per_token = (p.hq + p.hk) * per_head;
	const int64_t total = p.tokens * per_token;
	const int64_t stride = (int64_t)gridDim.x * kBlock;
	for (int64_t item = (int64_t)blockIdx.x * kBlock + threadIdx.x; item < total; item += stride) {
		const int64_t t = item / per_token;
		const int64_t pos = p.pos0 + t;
		if (pos == 0)
			continue;
		const int r = (int)(item - t * per_token);
		const int h = r / per_head;
		const int j = (r - h * per_head) * P;
		float *hb = h < p.hq ? p.q + (t * p.hq + h) * (int64_t)(2 * p.half) : p.k + (t * p.hk + (h - p.hq)) * (int64_t)(2 * p.half);
		const float *cr = p.cos_t + pos * p.rope_max_dim + j;
		const float *sr = p.sin_t + pos * p.rope_max_dim + j;
		if (VEC) {
			float4 *lo4 = reinterpret_cast<float4 *>(hb + j);
			float4 *hi4 = reinterpret_cast<float4 *>(hb + p.half + j);
			const float4 lo = ld_stream4(lo4), hi = ld_stream4(hi4);
			const float4 c = __ldg(reinterpret_cast<const float4 *>(cr));
			const float4 s = __ldg(reinterpret_cast<const float4 *>(sr));
			float4 a, b;
			rotate(lo.x, hi.x, c.x, s.x, a.x, b.x);
			rotate(lo.y, hi.y, c.y, s.y, a.y, b.y);
			rotate(lo.z, hi.z, c.z, s.z, a.z, b.z);
			rotate(lo.w, hi.w, c.w, s.w, a.w, b.w);
			st_stream4(lo4, a);
			st_stream4(hi4, b);
		} else {
			float a, b;
			rotate(hb[j], hb[p.half + j], __ldg(cr), __ldg(sr), a, b);
			hb[j] = a;
			hb[p.half + j] = b;
		}
	}
}

// Up to `oversubscribe` x the blocks resident at once (at most work_blocks).
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

extern "C" int v7g_rope_only_rows(float *q, float *k, int64_t tokens, int n_q_heads, int n_kv_heads, int head_dim, const float *cos_table, const float *sin_table, int64_t pos0, int rope_max_dim, void *stream)
{
	const char *what = "v7g_rope_only_rows";
	if (head_dim < 32 || head_dim > 1024 || head_dim % 32 != 0)
		return set_error(V7G_ERR_ARG, "%s: head_dim = %d must be a multiple of 32 in [32, 1024]", what, head_dim);
	if (tokens < 0 || n_q_heads < 0 || n_kv_heads < 0 || pos0 < 0 || rope_max_dim < 0)
		return set_error(V7G_ERR_ARG, "%s: negative tokens, head count, pos0 or rope_max_dim", what);
	if ((n_q_heads > 0 && !q) || (n_kv_heads > 0 && !k))
		return set_error(V7G_ERR_ARG, "%s: NULL tensor for a non-empty head set", what);
	const bool rotates = tokens > 1 || pos0 > 0;
	if (rotates && (!cos_table || !sin_table))
		return set_error(V7G_ERR_ARG, "%s: NULL cos/sin table", what);
	if (tokens == 0 || n_q_heads + n_kv_heads == 0 || !rotates)
		return clear_error();
	const int half = head_dim / 2;
	RopeOnlyArgs a{q, k, cos_table, sin_table, tokens, pos0, n_q_heads, n_kv_heads, half, rope_max_dim};
	const bool vec = (n_q_heads == 0 || aligned16(q)) && (n_kv_heads == 0 || aligned16(k)) && aligned16(cos_table) && aligned16(sin_table) && rope_max_dim % 4 == 0;
	const int64_t per_token = (int64_t)(n_q_heads + n_kv_heads) * (vec ? half / 4 : half);
	const int64_t blocks = (tokens * per_token + kBlock - 1) / kBlock;
	if (vec)
		return launch_persistent(k_rope_only_rows<true>, what, blocks, 4, stream, a);
	return launch_persistent(k_rope_only_rows<false>, what, blocks, 4, stream, a);
}
