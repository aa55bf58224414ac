// runtime.cu -- error reporting, launch accounting and device checks shared by
// every entry point of the library.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "internal.h"

namespace v7g {

namespace {
thread_local char t_error[512] = "";
std::atomic<uint64_t> g_launches{0};
// launch overlap: on unless the environment says V7G_LAUNCH_OVERLAP=0 (read
// once, when the library is loaded); v7g_set_launch_overlap changes it later
int overlap_from_env()
{
	const char *v = std::getenv("V7G_LAUNCH_OVERLAP");
	return (v && v[0] == '0' && v[1] == 0) ? 0 : 1;
}
std::atomic<int> g_launch_overlap{overlap_from_env()};

constexpr int kMaxDevices = 64;
struct CachedDevice {
	bool valid;
	DeviceInfo info;
};
CachedDevice g_devices[kMaxDevices];
std::mutex g_device_mutex;
} // namespace

int set_error(int code, const char *fmt, ...)
{
	va_list ap;
	va_start(ap, fmt);
	vsnprintf(t_error, sizeof(t_error), fmt, ap);
	va_end(ap);
	return code;
}

int clear_error()
{
	t_error[0] = 0;
	return V7G_OK;
}

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int current_device(DeviceInfo *out)
{
	int dev = 0;
	cudaError_t e = cudaGetDevice(&dev);
	if (e != cudaSuccess)
		return set_error(V7G_ERR_NO_DEVICE, "no CUDA device: %s", cudaGetErrorString(e));
	if (dev < 0 || dev >= kMaxDevices)
		return set_error(V7G_ERR_NO_DEVICE, "device ordinal %d out of range", dev);
	std::lock_guard<std::mutex> lock(g_device_mutex);
	CachedDevice &c = g_devices[dev];
	if (!c.valid) {
		cudaDeviceProp prop;
		e = cudaGetDeviceProperties(&prop, dev);
		if (e != cudaSuccess)
			return set_error(V7G_ERR_NO_DEVICE, "cudaGetDeviceProperties(%d): %s", dev, cudaGetErrorString(e));
		if (prop.major != 10)
			return set_error(V7G_ERR_NO_DEVICE, "device %d (%s) is sm_%d%d; this library is built for sm_100a only", dev, prop.name, prop.major, prop.minor);
		c.info.device = dev;
		c.info.sm_count = prop.multiProcessorCount;
		c.info.major = prop.major;
		c.info.minor = prop.minor;
		c.valid = true;
	}
	*out = c.info;
	return V7G_OK;
}

int check_launch(const char *what)
{
	cudaError_t e = cudaGetLastError();
	if (e != cudaSuccess)
		return set_error(V7G_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
	count_launch();
	return clear_error();
}

int check_launch(const char *what, cudaError_t launched)
{
	cudaError_t e = cudaGetLastError(); // clears a sticky error the launch left as well
	if (launched != cudaSuccess)
		e = launched;
	if (e != cudaSuccess)
		return set_error(V7G_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
	count_launch();
	return clear_error();
}

bool launch_overlap() { return g_launch_overlap.load(std::memory_order_relaxed) != 0; }

int resident_grid(const void *kernel, int block, size_t smem, int64_t work_blocks, const DeviceInfo &dev)
{
	int per_sm = 0;
	if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, block, smem) != cudaSuccess || per_sm < 1)
		per_sm = 1;
	int64_t cap = (int64_t)per_sm * dev.sm_count;
	int64_t g = work_blocks < cap ? work_blocks : cap;
	return g < 1 ? 1 : (int)g;
}

} // namespace v7g

namespace {
float g_rms_eps = 0.0f;
}

extern "C" {

void v7g_set_rms_eps(float eps) { g_rms_eps = eps; }
float v7g_get_rms_eps(void) { return g_rms_eps; }
float *v7g_rms_eps_slot(void) { return &g_rms_eps; }
const char *v7g_last_error(void) { return v7g::t_error; }
uint64_t v7g_launch_count(void) { return v7g::g_launches.load(std::memory_order_relaxed); }
void v7g_set_launch_overlap(int on) { v7g::g_launch_overlap.store(on ? 1 : 0, std::memory_order_relaxed); }
int v7g_get_launch_overlap(void) { return v7g::g_launch_overlap.load(std::memory_order_relaxed); }
const char *v7g_version(void) { return "v7g 0.1.0 (sm_100a; reference ABI cpki-gmbh/v7multiplikator v2.36.8)"; }

} // extern "C"
