// launch.cuh -- kernel launches that overlap the previous kernel's drain
// (programmatic dependent launch, sm_90 and later).
//
// A kernel launched with the programmatic-serialization attribute may be
// scheduled before the kernel ahead of it in the stream has finished: once
// every CTA of that kernel has started and executed
// griddepcontrol.launch_dependents (or exited), this kernel's CTAs take the
// SM slots the last wave frees, and each blocks in griddepcontrol.wait until
// the kernel ahead has completed and its memory operations are visible.  The
// launch, CTA rasterisation and the first instructions then run under the
// previous kernel's tail instead of after it: about 2 us per launch for a
// 100 MB streaming kernel issued back to back on B200 (18.5 -> 16.6 us).
//
// Every kernel of the library starts with kernel_entry(): the wait comes
// before its first global memory access, so stream order holds whatever the
// kernel ahead is (one of ours, a library's, or none: without the attribute,
// or behind a kernel that never triggers, the wait returns at once / the
// launch happens at that kernel's exit).  The trigger follows at once: the
// next kernel can only be scheduled after this grid's last CTA has started,
// so its CTAs never take a slot this grid still needs.  Neither instruction
// waits on anything but the kernel ahead's completion, which needs nothing
// from this grid, so no order of events deadlocks.
#pragma once
#include <utility>

#include "internal.h"

namespace v7g {

__device__ __forceinline__ void kernel_entry()
{
	asm volatile("griddepcontrol.wait;" ::: "memory");
	asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// kernel<<<grid, block, smem, stream>>>(args...) with the programmatic
// serialization attribute while launch overlap is on (v7g_set_launch_overlap).
// Returns the launch's own status.
template <typename... Params, typename... Args>
cudaError_t launch_kernel(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, void *stream, Args &&...args)
{
	cudaLaunchAttribute attr[1];
	attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
	attr[0].val.programmaticStreamSerializationAllowed = 1;
	cudaLaunchConfig_t cfg = {};
	cfg.gridDim = grid;
	cfg.blockDim = block;
	cfg.dynamicSmemBytes = smem;
	cfg.stream = static_cast<cudaStream_t>(stream);
	cfg.attrs = attr;
	cfg.numAttrs = launch_overlap() ? 1 : 0;
	return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

} // namespace v7g
