// abi.cpp -- the reference's export surface (include/v7_threading.h) on top of
// the batched device kernels.
//
// The reference's loader (src/v7_lib.h:585-739) resolves 99 names and calls
// them with the Microsoft x64 convention.  The hot-path entries here take one
// vector (or one token) per call, like the reference, and accept host or
// device memory for every pointer independently:
//   - a device (or managed) pointer is handed to the kernel as is;
//   - a host pointer is staged through a per-device workspace: inputs copied
//     in, outputs copied back before the call returns.
// Each call runs on a library-owned stream and returns with its results in
// place (the reference's calls are synchronous).  The reference's calls take
// no stream, so when any pointer is device memory the call first waits for
// all work already queued on that device (cudaDeviceSynchronize): a kernel of
// the caller's that is still writing an input, on any stream, has finished
// before the library reads it.  The calling thread's current device is the
// same after the call as before it.  A contract violation or a
// CUDA failure marks the engine dead with a reason (v7_engine_is_dead /
// v7_get_death_reason, src/v7_lib.h:179-184) and leaves the outputs unwritten,
// where the reference would FATAL (engine_landing.inc:150) or silently
// mis-size (rmsnorm_kernel.inc:15-19).
#include <cstdarg>
#include <cstddef>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/v7_threading.h"
#include "../../include/v7g.h"
#include "internal.h"

extern "C" float *v7g_rms_eps_slot(void);

unsigned long long v7g_zero_block[16];
int enable_token_dump = 0;
int enable_dump = 0;
// The reference sets this from its CPUID probe; this library needs no CPU
// feature, so it is 1.  A CUDA device is checked on the first kernel call.
int cpu_features_ok = 1;

namespace {

std::mutex g_mutex; // serialises the reference-ABI entries (shared workspace)
int g_dead = 0;
char g_reason[512] = "";

void die(const char *fmt, ...)
{
	va_list ap;
	va_start(ap, fmt);
	vsnprintf(g_reason, sizeof(g_reason), fmt, ap);
	va_end(ap);
	g_dead = 1;
}

// ---- per-device stream and staging workspace ------------------------------
struct DeviceCtx {
	cudaStream_t stream = nullptr;
	char *work = nullptr;
	size_t work_bytes = 0;
	// RoPE tables built by v7s_rope_init: [V7G_ROPE_TABLE_POSITIONS, rope_half]
	float *rope_cos = nullptr;
	float *rope_sin = nullptr;
	int rope_half = 0;
};
int g_fused_pos = 0;      // v7s_set_fused_rope
int g_fused_head_dim = 0; // v7s_set_fused_rope / v7s_rope_init
constexpr int kMaxDevices = 64;
DeviceCtx g_ctx[kMaxDevices];

int ensure_ctx(int dev, size_t bytes, DeviceCtx **out)
{
	if (dev < 0 || dev >= kMaxDevices)
		return -1;
	DeviceCtx &c = g_ctx[dev];
	if (!c.stream && cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking) != cudaSuccess)
		return -1;
	if (bytes > c.work_bytes) {
		if (c.work)
			cudaFree(c.work);
		c.work = nullptr;
		c.work_bytes = 0;
		size_t want = bytes < (1u << 20) ? (1u << 20) : bytes + bytes / 4;
		if (cudaMalloc(&c.work, want) != cudaSuccess) {
			cudaGetLastError();
			return -1;
		}
		c.work_bytes = want;
	}
	*out = &c;
	return 0;
}

// Classifies a pointer: 1 = device/managed memory (sets *dev), 0 = host.
int pointer_device(const void *p, int *dev)
{
	cudaPointerAttributes a;
	if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
		cudaGetLastError(); // plain host memory on old runtimes reports an error
		return 0;
	}
	if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) {
		*dev = a.device;
		return 1;
	}
	return 0;
}

// Maps every argument of one call to device memory.
class Stager {
  public:
	Stager()
	{
		if (cudaGetDevice(&caller_device_) != cudaSuccess) {
			cudaGetLastError();
			caller_device_ = -1;
		}
	}
	// The caller's current device again, whatever the call selected.
	~Stager()
	{
		int cur = -1;
		if (caller_device_ >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != caller_device_)
			cudaSetDevice(caller_device_);
		cudaGetLastError();
	}
	Stager(const Stager &) = delete;
	Stager &operator=(const Stager &) = delete;

	struct Arg {
		void *user;
		size_t bytes;
		bool in, out, host;
		size_t offset; // into the workspace, for host arguments
		int alias;     // index of an earlier identical host argument, or -1
	};

	int add(void *p, size_t bytes, bool in, bool out)
	{
		Arg a{p, bytes, in, out, true, 0, -1};
		int dev = -1;
		if (p && pointer_device(p, &dev)) {
			a.host = false;
			if (device_ < 0)
				device_ = dev;
			else if (device_ != dev)
				mixed_ = true;
		}
		if (a.host)
			for (size_t i = 0; i < args_.size(); ++i)
				if (args_[i].host && args_[i].user == p && args_[i].bytes == bytes) {
					a.alias = (int)i;
					args_[i].in = args_[i].in || in;
					args_[i].out = args_[i].out || out;
				}
		args_.push_back(a);
		return (int)args_.size() - 1;
	}

	// Selects the device, reserves the workspace and uploads host inputs.
	bool begin(const char *what)
	{
		what_ = what;
		if (mixed_) {
			die("%s: pointers on different CUDA devices", what);
			return false;
		}
		if (device_ < 0 && cudaGetDevice(&device_) != cudaSuccess) {
			cudaGetLastError();
			die("%s: no CUDA device", what);
			return false;
		}
		if (cudaSetDevice(device_) != cudaSuccess) {
			cudaGetLastError();
			die("%s: cannot select CUDA device %d", what, device_);
			return false;
		}
		// a device pointer may still be written by the caller's own queued
		// work, on a stream this call cannot know: wait for the whole device
		bool any_device = false;
		for (const Arg &a : args_)
			any_device = any_device || (a.user && !a.host);
		if (any_device && cudaDeviceSynchronize() != cudaSuccess)
			return fail("waiting for the caller's queued work");
		size_t total = 0;
		for (Arg &a : args_)
			if (a.host && a.alias < 0) {
				a.offset = total;
				total += (a.bytes + 255) & ~(size_t)255;
			}
		if (ensure_ctx(device_, total, &ctx_) != 0) {
			die("%s: cannot allocate a %zu-byte staging workspace on device %d", what, total, device_);
			return false;
		}
		for (Arg &a : args_)
			if (a.host && a.alias < 0 && a.in && a.bytes)
				if (cudaMemcpyAsync(ctx_->work + a.offset, a.user, a.bytes, cudaMemcpyHostToDevice, ctx_->stream) != cudaSuccess)
					return fail("host-to-device copy");
		return true;
	}

	// Device memory of `bytes` in the call's workspace, tied to no argument
	// (valid after begin()).
	int reserve(size_t bytes)
	{
		args_.push_back(Arg{nullptr, bytes, false, false, true, 0, -1});
		return (int)args_.size() - 1;
	}

	void *dev(int i) const
	{
		const Arg &a = args_[i];
		if (!a.host)
			return a.user;
		const Arg &b = a.alias >= 0 ? args_[a.alias] : a;
		return ctx_->work + b.offset;
	}

	cudaStream_t stream() const { return ctx_->stream; }

	// Checks the kernel status, copies host outputs back and waits.
	bool end(int rc)
	{
		if (rc != V7G_OK) {
			cudaStreamSynchronize(ctx_->stream);
			die("%s: %s", what_, v7g_last_error());
			return false;
		}
		for (const Arg &a : args_)
			if (a.host && a.alias < 0 && a.out && a.bytes)
				if (cudaMemcpyAsync(a.user, ctx_->work + a.offset, a.bytes, cudaMemcpyDeviceToHost, ctx_->stream) != cudaSuccess)
					return fail("device-to-host copy");
		if (cudaStreamSynchronize(ctx_->stream) != cudaSuccess)
			return fail("stream synchronisation");
		return true;
	}

  private:
	// Records the failure; copies already queued on the library stream use
	// the shared workspace, so they finish before the lock is released.
	bool fail(const char *step)
	{
		cudaError_t e = cudaGetLastError();
		die("%s: %s failed: %s", what_, step, cudaGetErrorString(e));
		if (ctx_ && ctx_->stream)
			cudaStreamSynchronize(ctx_->stream);
		cudaGetLastError();
		return false;
	}

	std::vector<Arg> args_;
	int caller_device_ = -1;
	int device_ = -1;
	bool mixed_ = false;
	DeviceCtx *ctx_ = nullptr;
	const char *what_ = "";
};

// ---- key store (the reference's MicroDB surface, reduced to a map) ---------
std::unordered_map<std::string, std::vector<unsigned char>> g_store;
int g_readonly = 0;
const char *kEpsKey = "__sys_rms_eps";
const char kDbMagic[8] = {'V', '7', 'G', 'D', 'B', '0', '0', '1'};

int store_add(const char *key, const void *data, unsigned long long len)
{
	if (!key || (!data && len))
		return 0;
	if (strcmp(key, kEpsKey) == 0) {
		if (len != sizeof(float))
			return 0;
		memcpy(v7g_rms_eps_slot(), data, sizeof(float));
		return 1;
	}
	if (g_readonly)
		return 0;
	const unsigned char *d = static_cast<const unsigned char *>(data);
	g_store[key].assign(d, d + len);
	return 1;
}

void *store_find(const char *key, unsigned long long *out_len)
{
	if (!key)
		return nullptr;
	if (strcmp(key, kEpsKey) == 0) {
		if (out_len)
			*out_len = sizeof(float);
		return v7g_rms_eps_slot();
	}
	auto it = g_store.find(key);
	if (it == g_store.end())
		return nullptr;
	if (out_len)
		*out_len = it->second.size();
	return it->second.empty() ? (void *)v7g_zero_block : it->second.data();
}

int store_save(const char *path)
{
	if (!path)
		return 0;
	FILE *f = fopen(path, "wb");
	if (!f)
		return 0;
	bool ok = fwrite(kDbMagic, 1, 8, f) == 8;
	float eps = *v7g_rms_eps_slot();
	auto put = [&](const std::string &k, const void *d, unsigned long long n) {
		unsigned int kl = (unsigned int)k.size();
		ok = ok && fwrite(&kl, 4, 1, f) == 1 && fwrite(k.data(), 1, kl, f) == kl && fwrite(&n, 8, 1, f) == 1 && (n == 0 || fwrite(d, 1, n, f) == n);
	};
	put(kEpsKey, &eps, sizeof(float));
	for (const auto &kv : g_store)
		put(kv.first, kv.second.data(), kv.second.size());
	ok = (fclose(f) == 0) && ok;
	return ok ? 1 : 0;
}

// Returns 1 on success, 0 when the file is missing, -1 when it is not a
// store written by store_save.
int store_load(const char *path)
{
	FILE *f = path ? fopen(path, "rb") : nullptr;
	if (!f)
		return 0;
	char magic[8];
	if (fread(magic, 1, 8, f) != 8 || memcmp(magic, kDbMagic, 8) != 0) {
		fclose(f);
		return -1;
	}
	std::unordered_map<std::string, std::vector<unsigned char>> loaded;
	float eps = *v7g_rms_eps_slot();
	bool ok = true;
	for (;;) {
		unsigned int kl;
		if (fread(&kl, 4, 1, f) != 1)
			break;
		std::string k(kl, '\0');
		unsigned long long n;
		if (kl > (1u << 20) || fread(&k[0], 1, kl, f) != kl || fread(&n, 8, 1, f) != 1 || n > (1ull << 40)) {
			ok = false;
			break;
		}
		std::vector<unsigned char> d(n);
		if (n && fread(d.data(), 1, n, f) != n) {
			ok = false;
			break;
		}
		if (k == kEpsKey && n == sizeof(float))
			memcpy(&eps, d.data(), sizeof(float));
		else
			loaded[k] = std::move(d);
	}
	fclose(f);
	if (!ok)
		return -1;
	g_store.swap(loaded);
	*v7g_rms_eps_slot() = eps;
	return 1;
}

} // namespace

extern "C" {

// ---- hot path --------------------------------------------------------------

V7_ABI void v7s_rmsnorm(float *o, float *x, float *weight, int size)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	if (size <= 0 || size % 32 != 0) {
		die("v7s_rmsnorm: size %d breaks the contract size > 0, size %% 32 == 0", size);
		return;
	}
	const size_t b = (size_t)size * sizeof(float);
	Stager s;
	int io = s.add(o, b, false, true), ix = s.add(x, b, true, false), iw = s.add(weight, b, true, false);
	if (!s.begin("v7s_rmsnorm"))
		return;
	s.end(v7g_rmsnorm_rows((float *)s.dev(io), (const float *)s.dev(ix), (const float *)s.dev(iw), 1, size, *v7g_rms_eps_slot(), s.stream()));
}

V7_ABI void v7s_add_inplace(float *x, float *y, int n)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	if (n <= 0 || n % 32 != 0) {
		die("v7s_add_inplace: n %d breaks the contract n > 0, n %% 32 == 0", n);
		return;
	}
	const size_t b = (size_t)n * sizeof(float);
	Stager s;
	int ix = s.add(x, b, true, true), iy = s.add(y, b, true, false);
	if (!s.begin("v7s_add_inplace"))
		return;
	s.end(v7g_add_inplace((float *)s.dev(ix), (const float *)s.dev(iy), n, s.stream()));
}

V7_ABI void v7s_fused_add_rmsnorm(float *o, float *residual, float *add, float *weight, int dim)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	if (dim < 0 || dim % 8 != 0) {
		die("v7s_fused_add_rmsnorm: dim %d breaks the contract dim %% 8 == 0", dim);
		return;
	}
	if (dim == 0)
		return;
	const size_t b = (size_t)dim * sizeof(float);
	Stager s;
	int io = s.add(o, b, false, true), ir = s.add(residual, b, true, true), ia = s.add(add, b, true, false), iw = s.add(weight, b, true, false);
	if (!s.begin("v7s_fused_add_rmsnorm"))
		return;
	s.end(v7g_fused_add_rmsnorm_rows((float *)s.dev(io), (float *)s.dev(ir), (const float *)s.dev(ia), (const float *)s.dev(iw), 1, dim, *v7g_rms_eps_slot(), s.stream()));
}

V7_ABI void v7s_rmsnorm_rope_heads(float *buf, int n_heads, int head_dim, float *norm_weight, float *cos_table, float *sin_table, int pos, int rope_max_dim)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	if (n_heads < 0 || head_dim < 32 || head_dim > 1024 || head_dim % 32 != 0 || pos < 0 || rope_max_dim < 0) {
		die("v7s_rmsnorm_rope_heads: n_heads %d, head_dim %d, pos %d, rope_max_dim %d break the contract (head_dim %% 32 == 0, 32 <= head_dim <= 1024)", n_heads, head_dim, pos, rope_max_dim);
		return;
	}
	if (n_heads == 0)
		return;
	const size_t hb = (size_t)head_dim * sizeof(float);
	const size_t half_b = (size_t)(head_dim / 2) * sizeof(float);
	Stager s;
	int ib = s.add(buf, hb * (size_t)n_heads, true, true), iw = s.add(norm_weight, hb, true, false);
	// The reference pre-offsets the tables to row pos (rmsnorm_rope_dispatch.inc:28-33)
	// and reads head_dim/2 entries of it; only that row is staged.
	int ic = -1, is = -1;
	if (pos != 0) {
		ic = s.add(cos_table + (size_t)pos * rope_max_dim, half_b, true, false);
		is = s.add(sin_table + (size_t)pos * rope_max_dim, half_b, true, false);
	}
	if (!s.begin("v7s_rmsnorm_rope_heads"))
		return;
	// One token at position pos: the staged row is the table (row stride 0).
	const float *c = ic >= 0 ? (const float *)s.dev(ic) : nullptr;
	const float *sn = is >= 0 ? (const float *)s.dev(is) : nullptr;
	s.end(v7g_rmsnorm_rope_rows((float *)s.dev(ib), nullptr, 1, n_heads, 0, head_dim, (const float *)s.dev(iw), nullptr, c, sn, pos, 0, *v7g_rms_eps_slot(), s.stream()));
}

V7_ABI void v7d_q8(float *xout, v7_q8_tensor *x, v7_q8_tensor *w, int n, int d)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	if (!x || !w || n <= 0 || n % 64 != 0 || d < 0) {
		die("v7d_q8: n %d, d %d or a NULL tensor break the contract n %% 64 == 0", n, d);
		return;
	}
	if (d == 0)
		return;
	const size_t ng = (size_t)n / 64;
	Stager s;
	int io = s.add(xout, (size_t)d * sizeof(float), false, true);
	int ixq = s.add(x->q, (size_t)n, true, false), ixs = s.add(x->s, ng * sizeof(float), true, false);
	int iwq = s.add(w->q, (size_t)d * n, true, false), iws = s.add(w->s, (size_t)d * ng * sizeof(float), true, false);
	if (!s.begin("v7d_q8"))
		return;
	s.end(v7g_q8_gemv((float *)s.dev(io), (const int8_t *)s.dev(ixq), (const float *)s.dev(ixs), (const int8_t *)s.dev(iwq), (const float *)s.dev(iws), 1, n, d, s.stream()));
}

static_assert(sizeof(v7_q8_batch4_args) == 120 && offsetof(v7_q8_batch4_args, xq) == 32 && offsetof(v7_q8_batch4_args, xs) == 64 &&
                  offsetof(v7_q8_batch4_args, wq) == 96 && offsetof(v7_q8_batch4_args, ws) == 104 && offsetof(v7_q8_batch4_args, n) == 112 &&
                  offsetof(v7_q8_batch4_args, d) == 116,
              "v7_q8_batch4_args: the layout of src/q8_batch4.h:29-38");

// The four tokens are gathered into one [4, n] block (and the outputs come
// out of one [4, d] block) so that v7g_q8_gemv's four-token blocks stream the
// weights once.
static void q8_batch4(const char *what, const v7_q8_batch4_args *args)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	if (!args) {
		die("%s: NULL argument block", what);
		return;
	}
	const int n = (int)args->n, d = (int)args->d;
	bool ok = args->n > 0 && args->n % 64 == 0 && args->n <= 65536 && args->d <= 0x7fffffffu && args->wq && args->ws;
	for (int t = 0; t < 4; ++t)
		ok = ok && args->out[t] && args->xq[t] && args->xs[t];
	if (!ok) {
		die("%s: n %u, d %u or a NULL pointer break the contract n %% 64 == 0, n <= 65536", what, args->n, args->d);
		return;
	}
	if (d == 0)
		return;
	const size_t ng = (size_t)n / 64;
	Stager s;
	int io[4], ixq[4], ixs[4];
	for (int t = 0; t < 4; ++t) {
		io[t] = s.add(args->out[t], (size_t)d * sizeof(float), false, true);
		ixq[t] = s.add(const_cast<int8_t *>(args->xq[t]), (size_t)n, true, false);
		ixs[t] = s.add(const_cast<float *>(args->xs[t]), ng * sizeof(float), true, false);
	}
	const int iwq = s.add(const_cast<int8_t *>(args->wq), (size_t)d * n, true, false);
	const int iws = s.add(const_cast<float *>(args->ws), (size_t)d * ng * sizeof(float), true, false);
	const int gq = s.reserve(4 * (size_t)n), gs = s.reserve(4 * ng * sizeof(float)), go = s.reserve(4 * (size_t)d * sizeof(float));
	if (!s.begin(what))
		return;
	int8_t *xq4 = (int8_t *)s.dev(gq);
	float *xs4 = (float *)s.dev(gs), *out4 = (float *)s.dev(go);
	for (int t = 0; t < 4; ++t)
		if (cudaMemcpyAsync(xq4 + (size_t)t * n, s.dev(ixq[t]), (size_t)n, cudaMemcpyDeviceToDevice, s.stream()) != cudaSuccess ||
		    cudaMemcpyAsync(xs4 + (size_t)t * ng, s.dev(ixs[t]), ng * sizeof(float), cudaMemcpyDeviceToDevice, s.stream()) != cudaSuccess) {
			s.end(v7g::set_error(V7G_ERR_CUDA, "%s: gathering the activations: %s", what, cudaGetErrorString(cudaGetLastError())));
			return;
		}
	int rc = v7g_q8_gemv(out4, xq4, xs4, (const int8_t *)s.dev(iwq), (const float *)s.dev(iws), 4, n, d, s.stream());
	for (int t = 0; t < 4 && rc == V7G_OK; ++t)
		if (cudaMemcpyAsync(s.dev(io[t]), out4 + (size_t)t * d, (size_t)d * sizeof(float), cudaMemcpyDeviceToDevice, s.stream()) != cudaSuccess)
			rc = v7g::set_error(V7G_ERR_CUDA, "%s: scattering the outputs: %s", what, cudaGetErrorString(cudaGetLastError()));
	s.end(rc);
}

V7_ABI void v7s_q8_batch4(const v7_q8_batch4_args *args) { q8_batch4("v7s_q8_batch4", args); }
V7_ABI void v7d_q8_batch4(const v7_q8_batch4_args *args) { q8_batch4("v7d_q8_batch4", args); }

V7_ABI void v7d_swiglu(float *xout, v7_f32_tensor *x, v7_q8_tensor *gate_w, int n, int d, v7_q8_tensor *up_w)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	if (!x || !gate_w || !up_w || n <= 0 || n % 64 != 0 || d < 0) {
		die("v7d_swiglu: n %d, d %d or a NULL tensor break the contract n %% 64 == 0", n, d);
		return;
	}
	if (d == 0)
		return;
	const size_t ng = (size_t)n / 64;
	Stager s;
	int io = s.add(xout, (size_t)d * sizeof(float), false, true);
	int ix = s.add(x->data, (size_t)n * sizeof(float), true, false);
	int igq = s.add(gate_w->q, (size_t)d * n, true, false), igs = s.add(gate_w->s, (size_t)d * ng * sizeof(float), true, false);
	int iuq = s.add(up_w->q, (size_t)d * n, true, false), ius = s.add(up_w->s, (size_t)d * ng * sizeof(float), true, false);
	if (!s.begin("v7d_swiglu"))
		return;
	s.end(v7g_swiglu_f32q8_gemv((float *)s.dev(io), (const float *)s.dev(ix), (const int8_t *)s.dev(igq), (const float *)s.dev(igs), (const int8_t *)s.dev(iuq), (const float *)s.dev(ius), 1, n, d, s.stream()));
}

V7_ABI void v7d_swiglu_q8(float *xout, v7_q8_tensor *x, v7_q8_tensor *gate_w, int n, int d, v7_q8_tensor *up_w)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	if (!x || !gate_w || !up_w || n <= 0 || n % 64 != 0 || d < 0) {
		die("v7d_swiglu_q8: n %d, d %d or a NULL tensor break the contract n %% 64 == 0", n, d);
		return;
	}
	if (d == 0)
		return;
	const size_t ng = (size_t)n / 64;
	Stager s;
	int io = s.add(xout, (size_t)d * sizeof(float), false, true);
	int ixq = s.add(x->q, (size_t)n, true, false), ixs = s.add(x->s, ng * sizeof(float), true, false);
	int igq = s.add(gate_w->q, (size_t)d * n, true, false), igs = s.add(gate_w->s, (size_t)d * ng * sizeof(float), true, false);
	int iuq = s.add(up_w->q, (size_t)d * n, true, false), ius = s.add(up_w->s, (size_t)d * ng * sizeof(float), true, false);
	if (!s.begin("v7d_swiglu_q8"))
		return;
	s.end(v7g_swiglu_q8_gemv((float *)s.dev(io), (const int8_t *)s.dev(ixq), (const float *)s.dev(ixs), (const int8_t *)s.dev(igq), (const float *)s.dev(igs), (const int8_t *)s.dev(iuq), (const float *)s.dev(ius), 1, n, d, s.stream()));
}

V7_ABI void v7s_rope_only_heads(float *buf, int n_heads, int head_dim, float *cos_table, float *sin_table, int pos, int rope_max_dim)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	if (n_heads < 0 || head_dim < 32 || head_dim > 1024 || head_dim % 32 != 0 || pos < 0 || rope_max_dim < 0) {
		die("v7s_rope_only_heads: n_heads %d, head_dim %d, pos %d, rope_max_dim %d break the contract (head_dim %% 32 == 0, 32 <= head_dim <= 1024)", n_heads, head_dim, pos, rope_max_dim);
		return;
	}
	if (n_heads == 0 || pos == 0) // position 0 is the identity (rope_only_kernel.inc:13-14)
		return;
	const size_t half_b = (size_t)(head_dim / 2) * sizeof(float);
	Stager s;
	int ib = s.add(buf, (size_t)head_dim * sizeof(float) * (size_t)n_heads, true, true);
	int ic = s.add(cos_table + (size_t)pos * rope_max_dim, half_b, true, false);
	int is = s.add(sin_table + (size_t)pos * rope_max_dim, half_b, true, false);
	if (!s.begin("v7s_rope_only_heads"))
		return;
	s.end(v7g_rope_only_rows((float *)s.dev(ib), nullptr, 1, n_heads, 0, head_dim, (const float *)s.dev(ic), (const float *)s.dev(is), pos, 0, s.stream()));
}

V7_ABI void v7s_qk_fork_heads(const v7_qk_fork_args *a)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	if (!a) {
		die("v7s_qk_fork_heads: NULL descriptor");
		return;
	}
	const int head_dim = a->head_dim, heads = a->heads, pos = a->pos;
	if (heads < 0 || head_dim < 32 || head_dim > 1024 || head_dim % 32 != 0 || pos < 0) {
		die("v7s_qk_fork_heads: heads %d, head_dim %d, pos %d break the contract (head_dim %% 32 == 0, 32 <= head_dim <= 1024)", heads, head_dim, pos);
		return;
	}
	if (heads == 0)
		return;
	const size_t hb = (size_t)head_dim * sizeof(float);
	const size_t half_b = hb / 2;
	Stager s;
	int ib = s.add(a->buf, hb * (size_t)heads, true, true), iw = s.add(a->weight, hb, true, false);
	int ic = -1, is = -1;
	if (pos != 0) { // the descriptor's tables are already offset to the position's row
		ic = s.add(a->cos, half_b, true, false);
		is = s.add(a->sin, half_b, true, false);
	}
	if (!s.begin("v7s_qk_fork_heads"))
		return;
	const float *c = ic >= 0 ? (const float *)s.dev(ic) : nullptr;
	const float *sn = is >= 0 ? (const float *)s.dev(is) : nullptr;
	s.end(v7g_rmsnorm_rope_rows((float *)s.dev(ib), nullptr, 1, heads, 0, head_dim, (const float *)s.dev(iw), nullptr, c, sn, pos, 0, *v7g_rms_eps_slot(), s.stream()));
}

V7_ABI void v7d_quantize(char *out_q, float *in_x, float *out_s, int n)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	if (n < 0) {
		die("v7d_quantize: n %d < 0", n);
		return;
	}
	if (n == 0)
		return;
	const size_t groups = ((size_t)n + 63) / 64;
	Stager s;
	int iq = s.add(out_q, (size_t)n, false, true), ix = s.add(in_x, (size_t)n * sizeof(float), true, false), is = s.add(out_s, groups * sizeof(float), false, true);
	if (!s.begin("v7d_quantize"))
		return;
	s.end(v7g_quantize_rows((int8_t *)s.dev(iq), (float *)s.dev(is), (const float *)s.dev(ix), 1, n, s.stream()));
}

V7_ABI void v7s_rmsnorm_quantize(char *out_q, float *in_x, float *out_s, int n, float *weight)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	if (n <= 0 || n % 64 != 0) {
		die("v7s_rmsnorm_quantize: n %d breaks the contract n > 0, n %% 64 == 0", n);
		return;
	}
	const size_t b = (size_t)n * sizeof(float);
	Stager s;
	int iq = s.add(out_q, (size_t)n, false, true), ix = s.add(in_x, b, true, false), is = s.add(out_s, (size_t)(n / 64) * sizeof(float), false, true), iw = s.add(weight, b, true, false);
	if (!s.begin("v7s_rmsnorm_quantize"))
		return;
	s.end(v7g_rmsnorm_quantize_rows((int8_t *)s.dev(iq), (float *)s.dev(is), (const float *)s.dev(ix), (const float *)s.dev(iw), 1, n, *v7g_rms_eps_slot(), s.stream()));
}

// ---- runtime surface ---------------------------------------------------------

V7_ABI int v7_init(const char *db_path)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	g_dead = 0;
	g_reason[0] = 0;
	if (!db_path) {
		g_store.clear();
		return 1;
	}
	int rc = store_load(db_path);
	if (rc == 0) {
		die("v7_init: cannot open %s", db_path);
		return 0;
	}
	if (rc < 0)
		g_store.clear(); // a foreign database: the kernels need none of its keys
	return 1;
}

V7_ABI int v7_db_load(const char *path)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	return store_load(path) == 1 ? 1 : 0;
}
V7_ABI int v7_db_save(const char *path)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	return store_save(path);
}
V7_ABI int db_load(const char *filename) { return v7_db_load(filename); }
V7_ABI int db_save(const char *filename) { return v7_db_save(filename); }
V7_ABI int ht_add(const char *key, void *data, unsigned long long data_len, unsigned int persist)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	return store_add(key, data, data_len);
}
V7_ABI void *ht_find(const char *key, unsigned long long *out_len)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	return store_find(key, out_len);
}
V7_ABI int v7_db_add(const char *key, const void *data, int len, unsigned int persist)
{
	if (len < 0)
		return 0;
	return ht_add(key, const_cast<void *>(data), (unsigned long long)len, persist);
}
V7_ABI void *v7_db_find(const char *key, unsigned long long *out_len) { return ht_find(key, out_len); }
V7_ABI void ht_init(void)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	g_store.clear();
}
V7_ABI void ht_destroy(void) { ht_init(); }
V7_ABI void db_set_readonly(int flag) { g_readonly = flag != 0; }

V7_ABI int v7_engine_is_dead(void) { return g_dead; }
V7_ABI const char *v7_get_death_reason(void) { return g_reason; }
V7_ABI const char *v7_get_version(void) { return v7g_version(); }
V7_ABI int v7_get_console_width(void) { return 80; }
V7_ABI void v7_do_fatal(const char *message)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	die("%s", message ? message : "v7_do_fatal");
}

namespace {
// ht_find_or_fatal of the reference (a missing key is fatal): the value of a
// 4-byte key, or false with the engine marked dead.
bool find_key4(const char *key, void *out)
{
	unsigned long long len = 0;
	void *p = store_find(key, &len);
	if (!p || len < 4) {
		die("v7s_rope_init: key %s not found", key);
		return false;
	}
	memcpy(out, p, 4);
	return true;
}
} // namespace

// Frequencies on the host (x87, as the reference), the [131072, half] tables
// on the current device, kept for v7g_get_rope_tables and the engine's calls.
// Caller holds g_mutex.  Returns a v7g status with the error recorded.
int rope_init_locked(int head_dim, float base, int scaling, float factor, float high, float low, int orig)
{
	using v7g::set_error;
	if (head_dim <= 0 || head_dim % 2 != 0 || head_dim / 2 > 256)
		return set_error(V7G_ERR_ARG, "rope init: head_dim %d must be even and at most 512", head_dim);
	const int half = head_dim / 2;
	double freqs[256];
	int rc = v7g_rope_freqs(freqs, half, base, scaling, factor, high, low, orig);
	if (rc != V7G_OK)
		return rc;
	int dev = -1;
	DeviceCtx *c = nullptr;
	if (cudaGetDevice(&dev) != cudaSuccess || ensure_ctx(dev, 0, &c) != 0) {
		cudaGetLastError();
		return set_error(V7G_ERR_NO_DEVICE, "rope init: no CUDA device");
	}
	if (c->rope_half != half || !c->rope_cos) {
		cudaFree(c->rope_cos);
		cudaFree(c->rope_sin);
		c->rope_cos = c->rope_sin = nullptr;
		c->rope_half = 0;
		const size_t bytes = (size_t)V7G_ROPE_TABLE_POSITIONS * half * sizeof(float);
		if (cudaMalloc(&c->rope_cos, bytes) != cudaSuccess || cudaMalloc(&c->rope_sin, bytes) != cudaSuccess) {
			cudaGetLastError();
			cudaFree(c->rope_cos);
			c->rope_cos = nullptr;
			return set_error(V7G_ERR_CUDA, "rope init: cannot allocate the RoPE tables on device %d", dev);
		}
	}
	c->rope_half = 0; // unusable until the build below has finished
	rc = v7g_rope_tables(c->rope_cos, c->rope_sin, 0, V7G_ROPE_TABLE_POSITIONS, half, half, freqs, c->stream);
	if (rc != V7G_OK)
		return rc;
	cudaError_t e = cudaStreamSynchronize(c->stream);
	if (e != cudaSuccess) {
		cudaGetLastError();
		return set_error(V7G_ERR_CUDA, "rope init: table build failed: %s", cudaGetErrorString(e));
	}
	c->rope_half = half;
	return v7g::clear_error();
}

V7_ABI void v7s_rope_init(int head_dim, float rope_base)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	g_fused_head_dim = head_dim;
	float base, factor = 0, high = 0, low = 0;
	int type, orig = 0;
	if (!find_key4("__sys_rope_base", &base) || !find_key4("__sys_rope_type", &type))
		return;
	if (type == 1 && (!find_key4("__sys_rope_factor", &factor) || !find_key4("__sys_rope_high_freq_factor", &high) ||
	                  !find_key4("__sys_rope_low_freq_factor", &low) || !find_key4("__sys_rope_orig_max_pos", &orig)))
		return;
	if (rope_init_locked(head_dim, base, type == 1 ? 1 : 0, factor, high, low, orig) != V7G_OK)
		die("v7s_rope_init: %s", v7g_last_error());
}

int v7g_rope_init(int head_dim, float base, int scaling, float factor, float high_freq_factor, float low_freq_factor, int orig_max_pos)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	return rope_init_locked(head_dim, base, scaling, factor, high_freq_factor, low_freq_factor, orig_max_pos);
}

// The position and head size of the reference's fused QKV matmul (which
// this library does not provide) are recorded, nothing more.
V7_ABI void v7s_set_fused_rope(int pos, int head_dim)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	g_fused_pos = pos;
	g_fused_head_dim = head_dim;
}

int v7g_get_rope_tables(const float **cos_table, const float **sin_table, int *half)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	int dev = -1;
	if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices || g_ctx[dev].rope_half == 0) {
		cudaGetLastError();
		return v7g::set_error(V7G_ERR_ARG, "v7g_get_rope_tables: v7s_rope_init has built no tables on this device");
	}
	if (cos_table)
		*cos_table = g_ctx[dev].rope_cos;
	if (sin_table)
		*sin_table = g_ctx[dev].rope_sin;
	if (half)
		*half = g_ctx[dev].rope_half;
	return v7g::clear_error();
}
// Worker spin policy of the CPU pool: nothing spins on the GPU path.
V7_ABI void v7s_set_spin(int flag) {}
V7_ABI void v7s_enable_thinking(int on) {}
V7_ABI unsigned long long get_config_was_fixed(void) { return 0; }

// Parallel workers: the streaming multiprocessors of the current device.
V7_ABI int v7s_get_num_workers(void)
{
	int dev = 0, sms = 0;
	if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
		cudaGetLastError();
		return 0;
	}
	return sms;
}

// Releases the per-device streams and staging workspaces.
V7_ABI void v7s_shutdown(void)
{
	std::lock_guard<std::mutex> lock(g_mutex);
	int cur = -1;
	cudaGetDevice(&cur);
	for (int d = 0; d < kMaxDevices; ++d) {
		DeviceCtx &c = g_ctx[d];
		if (!c.stream && !c.work && !c.rope_cos)
			continue;
		cudaSetDevice(d);
		if (c.stream)
			cudaStreamSynchronize(c.stream);
		if (c.work)
			cudaFree(c.work);
		cudaFree(c.rope_cos);
		cudaFree(c.rope_sin);
		if (c.stream)
			cudaStreamDestroy(c.stream);
		c = DeviceCtx();
	}
	if (cur >= 0)
		cudaSetDevice(cur);
	cudaGetLastError();
}
V7_ABI void v7_shutdown(void) { v7s_shutdown(); }

// Console formatting belongs to the reference's runtime, not to this library.
V7_ABI int v7sprintf(char *buffer, int buf_size, const char *format, ...)
{
	if (buffer && buf_size > 0)
		buffer[0] = 0;
	std::lock_guard<std::mutex> lock(g_mutex);
	die("v7sprintf: not provided by v7g");
	return 0;
}

// ---- everything outside the kernel path ------------------------------------

#define V7G_DEFINE_VOID(name, params)                   \
	V7_ABI void name params                             \
	{                                                   \
		std::lock_guard<std::mutex> lock(g_mutex);      \
		die(#name ": not provided by v7g");             \
	}
#define V7G_DEFINE_RET(type, name, params, value)       \
	V7_ABI type name params                             \
	{                                                   \
		std::lock_guard<std::mutex> lock(g_mutex);      \
		die(#name ": not provided by v7g");             \
		return (type)(value);                           \
	}
V7G_STUBS_VOID(V7G_DEFINE_VOID)
V7G_STUBS_RET(V7G_DEFINE_RET)

} // extern "C"
