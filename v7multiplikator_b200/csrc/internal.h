// internal.h -- host-side plumbing shared by the kernel translation units.
#pragma once
#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

#include "../../include/v7g.h"

namespace v7g {

// Records `code` with a printf-style message as the calling thread's last
// error (v7g_last_error) and returns `code`.
int set_error(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
// Clears the calling thread's last error; returns V7G_OK.
int clear_error();

// Counts one kernel launch (v7g_launch_count).
void count_launch();

struct DeviceInfo {
	int device;
	int sm_count;
	int major;
	int minor;
};
// Properties of the current device, cached per device.  Fails with
// V7G_ERR_NO_DEVICE unless the device is compute capability 10.x, the only
// architecture this library carries code for.
int current_device(DeviceInfo *out);

// Checks the launch just issued; on failure records the CUDA error.
int check_launch(const char *what);
// The same for a launch that returned its own status (cudaLaunchKernelEx).
int check_launch(const char *what, cudaError_t launched);

// Whether kernels are launched to overlap the drain of the kernel ahead of
// them in the stream (v7g_set_launch_overlap; on by default).
bool launch_overlap();

// Persistent-grid size: at most `work_blocks` blocks, at most what fits
// resident on the device at once (occupancy of `kernel` at `block` threads).
int resident_grid(const void *kernel, int block, size_t smem, int64_t work_blocks, const DeviceInfo &dev);

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Given-up bounded waits of the row pipelines in norm.cu and norm_q8.cu
// (0xffffffff when the count cannot be read).
unsigned int norm_pipe_timeouts();
unsigned int norm_q8_pipe_timeouts();

} // namespace v7g
