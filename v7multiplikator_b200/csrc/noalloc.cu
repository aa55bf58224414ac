// noalloc.cu -- RMSNorm rows on host buffers through a fixed, load-time
// device buffer: an entry point that allocates no memory.
//
// The reference-ABI entries (v7s_rmsnorm & co.) accept host buffers by staging
// them through a device workspace the library obtains with cudaMalloc.  Some
// callers cannot let a library do that: a host program sharing the GPU with a
// framework whose caching allocator has already reserved nearly all device
// memory (the allocation fails or fragments that pool), a latency-critical
// loop that cannot afford the device-wide synchronisation cudaMalloc and
// cudaFree may impose, or a deployment whose policy forbids device
// allocations after start-up.  v7g_rmsnorm_rows_noalloc serves them: its
// staging area is the static array below, created with the module on every
// GPU that loads the library and held until the process exits.
//
// The array is shared by every call.  Calls are serialised on the host and
// each waits for its stream before returning -- on its failure paths too,
// once anything has been queued -- so two calls of this entry point never
// overlap on the GPU; anything else that made them overlap would race on the
// array.  Each call copies its whole input in and its whole output out, so
// the contents a previous call left behind are never read and nothing needs
// clearing.  The array's device address is looked up once per device and
// kept for the life of the process, so a cudaDeviceReset between calls is
// not supported; `stream` must belong to the current device.
#include <mutex>

#include "internal.h"

namespace v7g {
namespace {

constexpr size_t kScratchBytes = V7G_NOALLOC_SCRATCH_BYTES; // 4 MiB per GPU
constexpr size_t kAlign = 256;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_mutex;
unsigned char *g_scratch_addr[kMaxDevices]; // device address of the array, per device

size_t round_up(size_t v) { return (v + kAlign - 1) & ~(kAlign - 1); }

// Once per device, with that device current: the array's device address.  In
// host code the array's name is only a stand-in, never a usable pointer.
int scratch_for(int device, unsigned char **out)
{
	if (device < 0 || device >= kMaxDevices)
		return set_error(V7G_ERR_UNSUPPORTED, "v7g_rmsnorm_rows_noalloc: device %d beyond the %d tracked", device, kMaxDevices);
	if (!g_scratch_addr[device]) {
		void *p = nullptr;
		const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
		if (e != cudaSuccess) {
			cudaGetLastError();
			return set_error(V7G_ERR_CUDA, "v7g_rmsnorm_rows_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
		}
		g_scratch_addr[device] = static_cast<unsigned char *>(p);
	}
	*out = g_scratch_addr[device];
	return V7G_OK;
}

int cuda_fail(const char *step, cudaError_t e)
{
	cudaGetLastError();
	return set_error(V7G_ERR_CUDA, "v7g_rmsnorm_rows_noalloc: %s failed: %s", step, cudaGetErrorString(e));
}

// A failure after the first copy was queued: whatever is still queued on `s`
// reads or writes the shared array, so wait for it before the lock is
// released (the next call may use another stream).  Returns `rc`, keeping the
// first failure's message.
int drain_and_fail(cudaStream_t s, int rc)
{
	cudaStreamSynchronize(s);
	cudaGetLastError();
	return rc;
}

} // namespace
} // namespace v7g

using namespace v7g;

extern "C" int v7g_rmsnorm_rows_noalloc(float *o, const float *x, const float *w, int64_t rows, int n, float eps, void *stream)
{
	const char *what = "v7g_rmsnorm_rows_noalloc";
	if (n <= 0 || n % 32 != 0 || n >= (1 << 24))
		return set_error(V7G_ERR_ARG, "%s: n = %d must be a positive multiple of 32 below 2^24", what, n);
	if (rows < 0)
		return set_error(V7G_ERR_ARG, "%s: rows = %lld < 0", what, (long long)rows);
	if (rows == 0)
		return clear_error();
	if (!o || !x || !w)
		return set_error(V7G_ERR_ARG, "%s: NULL pointer", what);
	const size_t wb = (size_t)n * sizeof(float);
	if ((uint64_t)rows > (kScratchBytes / wb)) // keeps rows * n * 4 below from overflowing
		return set_error(V7G_ERR_ARG, "%s: %lld rows of %d floats exceed the %zu-byte static scratch", what, (long long)rows, n, kScratchBytes);
	const size_t xb = (size_t)rows * wb;
	const size_t need = round_up(wb) + 2 * round_up(xb);
	if (need > kScratchBytes)
		return set_error(V7G_ERR_ARG, "%s: %lld rows of %d floats need %zu bytes of staging, more than the %zu-byte static scratch (at most %zu floats of x and o together, plus gamma)",
		                 what, (long long)rows, n, need, kScratchBytes, (kScratchBytes - round_up(wb)) / sizeof(float));
	std::lock_guard<std::mutex> lock(g_mutex);
	DeviceInfo dev;
	int rc = current_device(&dev);
	if (rc != V7G_OK)
		return rc;
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	// the default streams (NULL, legacy, per-thread) are the current device's
	int stream_dev = dev.device;
	cudaError_t e = cudaSuccess;
	if (s && s != cudaStreamLegacy && s != cudaStreamPerThread) {
		e = cudaStreamGetDevice(s, &stream_dev);
		if (e != cudaSuccess)
			return cuda_fail("querying the stream's device", e);
	}
	if (stream_dev != dev.device)
		return set_error(V7G_ERR_ARG, "%s: the stream belongs to device %d, the current device is %d", what, stream_dev, dev.device);
	unsigned char *base = nullptr;
	rc = scratch_for(dev.device, &base);
	if (rc != V7G_OK)
		return rc;
	float *dw = reinterpret_cast<float *>(base);
	float *dx = reinterpret_cast<float *>(base + round_up(wb));
	float *dout = reinterpret_cast<float *>(base + round_up(wb) + round_up(xb));
	e = cudaMemcpyAsync(dw, w, wb, cudaMemcpyDefault, s);
	if (e != cudaSuccess)
		return drain_and_fail(s, cuda_fail("copying gamma in", e));
	e = cudaMemcpyAsync(dx, x, xb, cudaMemcpyDefault, s);
	if (e != cudaSuccess)
		return drain_and_fail(s, cuda_fail("copying x in", e));
	rc = v7g_rmsnorm_rows(dout, dx, dw, rows, n, eps, stream);
	if (rc != V7G_OK)
		return drain_and_fail(s, rc);
	e = cudaMemcpyAsync(o, dout, xb, cudaMemcpyDefault, s);
	if (e != cudaSuccess)
		return drain_and_fail(s, cuda_fail("copying o out", e));
	e = cudaStreamSynchronize(s);
	if (e != cudaSuccess)
		return cuda_fail("stream synchronisation", e);
	return clear_error();
}
