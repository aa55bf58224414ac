// norm.cu -- RMSNorm and fused residual-add + RMSNorm over rows of device
// memory, one warp per row.
//
// Lane l owns sum-of-squares chain l of the reference's 4 x 8 FMA accumulator
// layout (element e belongs to chain e % 32), reads its elements e = l + 32k
// with coalesced 128-byte warp accesses, keeps them in registers and writes
// the output from there: every activation is read once and written once.
// HBM-bound: bytes per row = 4n read + 4n written (+ 4n each for the residual
// of the fused add), gamma served from L1/L2.
#include "internal.h"
#include "reduce.cuh"

namespace v7g {
namespace {

constexpr int kBlock = 256;
constexpr int kWarpsPerBlock = kBlock / 32;

// --- A1  RMSNorm rows (rmsnorm_kernel.inc:12-75), caller's MXCSR: no FTZ ---
// CACHE = register slots per lane; rows longer than 32 * CACHE re-read the
// overflow elements in the output pass instead of holding them.
template <int CACHE>
__global__ void __launch_bounds__(kBlock) k_rmsnorm_rows(float *o, const float *x, const float *__restrict__ w, int64_t rows, int n, float eps)
{
	using M = F<false>;
	const int lane = threadIdx.x & 31;
	const int64_t nwarps = ((int64_t)gridDim.x * kBlock) >> 5;
	const int vpl = n >> 5;
	const float nf = (float)n;
	for (int64_t row = ((int64_t)blockIdx.x * kBlock + threadIdx.x) >> 5; row < rows; row += nwarps) {
		const float *xr = x + row * n + lane;
		float *orow = o + row * n + lane;
		float v[CACHE];
#pragma unroll
		for (int k = 0; k < CACHE; ++k)
			if (k < vpl)
				v[k] = ld_stream(xr + 32 * k);
		float acc = 0.0f;
#pragma unroll
		for (int k = 0; k < CACHE; ++k)
			if (k < vpl)
				acc = M::fma(v[k], v[k], acc);
		for (int k = CACHE; k < vpl; ++k) {
			float t = ld_stream(xr + 32 * k);
			acc = M::fma(t, t, acc);
		}
		const float scale = rms_scale<false>(reduce_chains_4x8<false>(acc), nf, eps);
#pragma unroll
		for (int k = 0; k < CACHE; ++k)
			if (k < vpl)
				st_stream(orow + 32 * k, M::mul(M::mul(v[k], scale), __ldg(w + lane + 32 * k)));
		for (int k = CACHE; k < vpl; ++k)
			st_stream(orow + 32 * k, M::mul(M::mul(ld_stream(xr + 32 * k), scale), __ldg(w + lane + 32 * k)));
	}
}

// --- A2  fused residual-add + RMSNorm rows (add_rmsnorm_kernel.inc:15-129) ---
// When n/8 is not a multiple of 4 the reference first folds the L = (n/8) % 4
// leading blocks into accumulator A (lanes 0..7 here), then runs the 4-way
// groups from block L on; chain lane l then covers e = 8L + l + 32k.
template <int CACHE>
__global__ void __launch_bounds__(kBlock) k_fused_add_rmsnorm_rows(float *o, float *res, const float *add, const float *__restrict__ w, int64_t rows, int n, float eps)
{
	using M = F<false>;
	const int lane = threadIdx.x & 31;
	const int64_t nwarps = ((int64_t)gridDim.x * kBlock) >> 5;
	const int left = (n >> 3) & 3;
	const int off = 8 * left;
	const int vpl = (n - off) >> 5;
	const float nf = (float)n;
	for (int64_t row = ((int64_t)blockIdx.x * kBlock + threadIdx.x) >> 5; row < rows; row += nwarps) {
		float *rr = res + row * n;
		const float *ar = add + row * n;
		float *orow = o + row * n;
		float acc = 0.0f;
		float pre[3] = {0.0f, 0.0f, 0.0f};
		if (left != 0 && lane < 8) {
#pragma unroll
			for (int b = 0; b < 3; ++b)
				if (b < left) {
					pre[b] = M::add(ld_stream(rr + 8 * b + lane), ld_stream(ar + 8 * b + lane));
					acc = M::fma(pre[b], pre[b], acc);
				}
		}
		float *rm = rr + off + lane;
		const float *am = ar + off + lane;
		float v[CACHE];
#pragma unroll
		for (int k = 0; k < CACHE; ++k)
			if (k < vpl)
				v[k] = M::add(ld_stream(rm + 32 * k), ld_stream(am + 32 * k));
#pragma unroll
		for (int k = 0; k < CACHE; ++k)
			if (k < vpl)
				acc = M::fma(v[k], v[k], acc);
		for (int k = CACHE; k < vpl; ++k) {
			float s = M::add(ld_stream(rm + 32 * k), ld_stream(am + 32 * k));
			rm[32 * k] = s; // read back in the output pass
			acc = M::fma(s, s, acc);
		}
		const float scale = rms_scale<false>(reduce_chains_4x8<false>(acc), nf, eps);
		if (left != 0 && lane < 8) {
#pragma unroll
			for (int b = 0; b < 3; ++b)
				if (b < left) {
					st_stream(rr + 8 * b + lane, pre[b]);
					st_stream(orow + 8 * b + lane, M::mul(M::mul(pre[b], scale), __ldg(w + 8 * b + lane)));
				}
		}
		float *om = orow + off + lane;
		const float *wm = w + off + lane;
#pragma unroll
		for (int k = 0; k < CACHE; ++k)
			if (k < vpl) {
				st_stream(rm + 32 * k, v[k]);
				st_stream(om + 32 * k, M::mul(M::mul(v[k], scale), __ldg(wm + 32 * k)));
			}
		for (int k = CACHE; k < vpl; ++k)
			st_stream(om + 32 * k, M::mul(M::mul(rm[32 * k], scale), __ldg(wm + 32 * k)));
	}
}

// Register budget: the smallest slot count that holds the row, up to 64
// (rows of up to 2048 floats stay entirely in registers).
int row_cache_slots(int vpl) { return vpl <= 8 ? 8 : vpl <= 16 ? 16 : vpl <= 32 ? 32 : 64; }

template <typename Kernel, typename... Args>
int launch_rows(Kernel kernel, const char *what, int64_t rows, void *stream, Args... args)
{
	DeviceInfo dev;
	int rc = current_device(&dev);
	if (rc != V7G_OK)
		return rc;
	const int64_t want = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
	const int grid = resident_grid((const void *)kernel, kBlock, 0, want, dev);
	kernel<<<grid, kBlock, 0, (cudaStream_t)stream>>>(args...);
	return check_launch(what);
}

bool row_len_ok(int n) { return n > 0 && n < (1 << 24); }

} // namespace
} // namespace v7g

using namespace v7g;

extern "C" {

int v7g_rmsnorm_rows(float *o, const float *x, const float *w, int64_t rows, int n, float eps, void *stream)
{
	if (!row_len_ok(n) || n % 32 != 0)
		return set_error(V7G_ERR_ARG, "v7g_rmsnorm_rows: n = %d must be a positive multiple of 32 below 2^24", n);
	if (rows < 0)
		return set_error(V7G_ERR_ARG, "v7g_rmsnorm_rows: rows = %lld < 0", (long long)rows);
	if (rows == 0)
		return clear_error();
	if (!o || !x || !w)
		return set_error(V7G_ERR_ARG, "v7g_rmsnorm_rows: NULL pointer");
	switch (row_cache_slots(n / 32)) {
	case 8:
		return launch_rows(k_rmsnorm_rows<8>, "v7g_rmsnorm_rows", rows, stream, o, x, w, rows, n, eps);
	case 16:
		return launch_rows(k_rmsnorm_rows<16>, "v7g_rmsnorm_rows", rows, stream, o, x, w, rows, n, eps);
	case 32:
		return launch_rows(k_rmsnorm_rows<32>, "v7g_rmsnorm_rows", rows, stream, o, x, w, rows, n, eps);
	default:
		return launch_rows(k_rmsnorm_rows<64>, "v7g_rmsnorm_rows", rows, stream, o, x, w, rows, n, eps);
	}
}

int v7g_fused_add_rmsnorm_rows(float *o, float *residual, const float *add, const float *w, int64_t rows, int n, float eps, void *stream)
{
	if (!row_len_ok(n) || n % 8 != 0)
		return set_error(V7G_ERR_ARG, "v7g_fused_add_rmsnorm_rows: n = %d must be a positive multiple of 8 below 2^24", n);
	if (rows < 0)
		return set_error(V7G_ERR_ARG, "v7g_fused_add_rmsnorm_rows: rows = %lld < 0", (long long)rows);
	if (rows == 0)
		return clear_error();
	if (!o || !residual || !add || !w)
		return set_error(V7G_ERR_ARG, "v7g_fused_add_rmsnorm_rows: NULL pointer");
	const int vpl = (n - 8 * ((n >> 3) & 3)) / 32;
	switch (row_cache_slots(vpl)) {
	case 8:
		return launch_rows(k_fused_add_rmsnorm_rows<8>, "v7g_fused_add_rmsnorm_rows", rows, stream, o, residual, add, w, rows, n, eps);
	case 16:
		return launch_rows(k_fused_add_rmsnorm_rows<16>, "v7g_fused_add_rmsnorm_rows", rows, stream, o, residual, add, w, rows, n, eps);
	case 32:
		return launch_rows(k_fused_add_rmsnorm_rows<32>, "v7g_fused_add_rmsnorm_rows", rows, stream, o, residual, add, w, rows, n, eps);
	default:
		return launch_rows(k_fused_add_rmsnorm_rows<64>, "v7g_fused_add_rmsnorm_rows", rows, stream, o, residual, add, w, rows, n, eps);
	}
}

} // extern "C"
