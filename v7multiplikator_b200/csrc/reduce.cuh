// reduce.cuh -- warp-level pieces shared by the row kernels.
#pragma once
#include "fp.cuh"

namespace v7g {

constexpr unsigned kFullMask = 0xffffffffu;

// Sum of squares in v7's order.  The reference accumulates a row with four
// 8-lane FMA accumulators, 8-float block b feeding accumulator b % 4
// (rmsnorm_kernel.inc:22-40), so element e lands in chain e % 32 and each chain
// runs over e = c, c+32, c+64, ... in order.  Lane l of a warp owns chain l, so
// the chains are computed exactly.  The merge (A+B)+(C+D)
// (rmsnorm_kernel.inc:43-45) and the HADD_YMM tree (v7_macros.inc:38-45) are a
// fixed pairwise tree over the 32 chains; lane l = 8*a + c holds accumulator a,
// lane c, so the tree is the butterfly 8, 16, 4, 1, 2.  fp32 addition is
// commutative, so every lane ends with the bit-identical total.
template <bool FTZ>
__device__ __forceinline__ float reduce_chains_4x8(float acc)
{
	using M = F<FTZ>;
	acc = M::add(acc, __shfl_xor_sync(kFullMask, acc, 8));
	acc = M::add(acc, __shfl_xor_sync(kFullMask, acc, 16));
	acc = M::add(acc, __shfl_xor_sync(kFullMask, acc, 4));
	acc = M::add(acc, __shfl_xor_sync(kFullMask, acc, 1));
	acc = M::add(acc, __shfl_xor_sync(kFullMask, acc, 2));
	return acc;
}

// COMPUTE_RMS_SCALE (v7_macros.inc:348-354): 1 / sqrt(ss / n + eps), every
// step one correctly rounded IEEE operation.
template <bool FTZ>
__device__ __forceinline__ float rms_scale(float ss, float nf, float eps)
{
	using M = F<FTZ>;
	return M::rcp(M::sqrt(M::add(M::div(ss, nf), eps)));
}

// One level of an x86 MAXPS tree across lanes: the lane whose `mask` bit is
// clear holds the first operand.  Reproduces the reference's NaN behaviour
// (MAXPS returns its second operand when either input is NaN).
__device__ __forceinline__ float max_tree_step(float v, int mask, int lane)
{
	float o = __shfl_xor_sync(kFullMask, v, mask);
	bool first = (lane & mask) == 0;
	float a = first ? v : o;
	float b = first ? o : v;
	return x86_max(a, b);
}

// Streaming global accesses: activations are touched once, so they are read
// and written with the evict-first policy and do not displace reused data
// (gamma, RoPE tables) from the caches.
__device__ __forceinline__ float ld_stream(const float *p) { return __ldcs(p); }
__device__ __forceinline__ float4 ld_stream4(const float4 *p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream(float *p, float v) { __stcs(p, v); }
__device__ __forceinline__ void st_stream4(float4 *p, float4 v) { __stcs(p, v); }

} // namespace v7g
