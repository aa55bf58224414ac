// pipeline.cuh -- shared-memory stage pipeline on sm_100: 1-D bulk copies
// (cp.async.bulk, the TMA engine without a tensor map) into shared memory,
// completed on transaction-counting mbarriers, and bounded waits.
//
// Every wait here gives up after kWaitLimit polls (seconds of wall time, far
// beyond any legitimate copy), counts the event in a device word the host can
// read, and returns false so the kernel can leave instead of hanging.  No
// copy uses cluster multicast.
#pragma once
#include <cstdint>

namespace v7g {

constexpr uint32_t kWaitLimit = 1u << 23;

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
	asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Makes barrier initialisation visible to the async (copy) proxy.
__device__ __forceinline__ void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

// Orders this thread's earlier generic-proxy shared-memory writes before
// later async-proxy (bulk copy) accesses to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes)
{
	asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
	asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Waits for the completion of the barrier phase with the given parity;
// false (and *timeouts incremented) when the bound ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, unsigned int *timeouts)
{
	const uint32_t a = smem_addr(bar);
	for (uint32_t i = 0; i < kWaitLimit; ++i) {
		uint32_t done;
		asm volatile("{\n\t.reg .pred p;\n\t"
		             "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
		             "selp.u32 %0, 1, 0, p;\n\t}"
		             : "=r"(done)
		             : "r"(a), "r"(parity)
		             : "memory");
		if (done)
			return true;
	}
	atomicAdd(timeouts, 1u);
	return false;
}

// Global -> shared bulk copy of `bytes` (a multiple of 16; both addresses
// 16-byte aligned), completing `bytes` transactions on `bar`.
__device__ __forceinline__ void bulk_copy_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
	asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
	             "l"(src), "r"(bytes), "r"(smem_addr(bar))
	             : "memory");
}

// Named barrier over `count` threads (a multiple of 32), id 1..15.
__device__ __forceinline__ void named_sync(int id, int count) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory"); }

} // namespace v7g
