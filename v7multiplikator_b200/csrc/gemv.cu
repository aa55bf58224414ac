// gemv.cu -- Q8-weight matrix-vector products: v7d_q8, v7d_swiglu_q8, the
// quantise-then-multiply v7d_q8_fused, and the fp32-activation v7d_swiglu.
//
// Arithmetic of the reference (q8_kernel.inc:22-201, swiglu_q8_kernel.inc:
// 16-286, swiglu_kernel.inc:30-249), reproduced bit for bit:
//   Q8 x Q8: per 64-element group, eight int32 "lane" dots -- lane l covers
//     bytes 4l..4l+3 of the group's low 32 bytes and 4l..4l+3 of its high 32
//     (vpmaddubsw / vpmaddwd / vpaddd); each converted to float (exact), the
//     weight scale times the activation scale rounded once, one fused
//     multiply-add per lane into eight lane accumulators; at the end the
//     HADD_YMM tree (l_j + l_{j+4}, then (t0 + t1) + (t2 + t3)).
//   F32 x Q8 (dual-row path): per element e, w_e converted to float times its
//     group scale (rounded), fused multiply-add with x_e into lane e % 8 of
//     one accumulator; HADD_YMM at the end.
//   SwiGLU epilogue: (sigmoid(g) * g) * u with EVAL_SIGMOID.  FTZ+DAZ
//   throughout (the reference runs these on its dispatched workers).
//
// The lane accumulators are eight independent fp32 chains per output row, so
// the GPU runs one chain per thread: eight threads per row, four rows per
// warp.  A thread streams its row's bytes 4l..4l+3 and 32+4l..32+4l+3 of every
// group (two 4-byte loads per matrix; the row's eight threads read both
// 32-byte sectors of the group whole) and its dp4a dot; the activation codes
// and scales are staged once per CTA in shared memory.  Loads for kUnroll
// groups are issued before their arithmetic.  The weights are read exactly
// once: HBM-bound at d x n x (1 + 4/64) bytes per matrix.
#include "internal.h"
#include "q8.cuh"

namespace v7g {
namespace {

constexpr int kBlock = 256;
constexpr int kLanes = 8;                     // HADD_YMM lanes per row
constexpr int kRowsPerBlock = kBlock / kLanes; // 32
constexpr int kUnroll = 8;                    // groups loaded ahead of their arithmetic
constexpr int kMaxN = 65536;                  // activation staged in shared memory

// The weight bytes the reference's vpsignb cannot negate: a -128 weight
// against a negative activation contributes |a| * (-128) there instead of
// a * (-128), i.e. 256 * a more than the true product.  The exporter never
// writes -128 (swiglu_q8_kernel.inc:17-23), so this runs only on inputs
// outside that contract.
__device__ __noinline__ int neg128_correction(uint32_t a, uint32_t w)
{
	int c = 0;
#pragma unroll
	for (int k = 0; k < 4; ++k) {
		const int ab = (int)(int8_t)(a >> (8 * k));
		const uint32_t wb = (w >> (8 * k)) & 0xffu;
		if (wb == 0x80u && ab < 0)
			c += 256 * ab;
	}
	return c;
}

// Non-zero when a byte of w is 0x80 (-128).
__device__ __forceinline__ uint32_t has_neg128(uint32_t w)
{
	const uint32_t t = w ^ 0x80808080u;
	return (t - 0x01010101u) & ~t & 0x80808080u;
}

// One lane's dot over one group: the low word and the high word.
__device__ __forceinline__ int lane_dot(uint32_t a_lo, uint32_t w_lo, uint32_t a_hi, uint32_t w_hi)
{
	int d = __dp4a((int)a_hi, (int)w_hi, __dp4a((int)a_lo, (int)w_lo, 0));
	if (has_neg128(w_lo) | has_neg128(w_hi))
		d += neg128_correction(a_lo, w_lo) + neg128_correction(a_hi, w_hi);
	return d;
}

// HADD_YMM over the row's eight lane threads (consecutive lanes of a warp):
// (l_j + l_{j+4}), then (t0 + t1) + (t2 + t3); the sum lands in lane j = 0.
__device__ __forceinline__ float hadd_lanes(float v)
{
	using M = F<true>;
	v = M::add(v, __shfl_xor_sync(0xffffffffu, v, 4));
	v = M::add(v, __shfl_xor_sync(0xffffffffu, v, 1));
	return M::add(v, __shfl_xor_sync(0xffffffffu, v, 2));
}

struct GemvArgs {
	float *out;            // [batch, d]
	const int8_t *xq;      // [batch, n] codes (Q8 activation)
	const float *xs;       // [batch, n/64]
	const float *xf;       // [batch, n] fp32 activation (fused quantise, F32 x Q8)
	const int8_t *wq[2];   // gate (or the only matrix), up: [d, n]
	const float *ws[2];    // [d, n/64]
	int n, d;
};

// Quantise the CTA's activation row into shared memory with v7d_quantize's
// rules (quantize_kernel.inc:43-106): half a warp per 64-element group, one
// float4 per lane.
__device__ void stage_quantized(const float *x, int n, uint32_t *sq, float *ss)
{
	const int lane = threadIdx.x & 31, half = lane >> 4, hl = lane & 15;
	const int groups = n / kQ8Group;
	const bool vec = (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
	for (int g = (threadIdx.x >> 5) * 2 + half; g - half < groups; g += (kBlock / 32) * 2) {
		float4 h = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
		if (g < groups) {
			const float *p = x + (int64_t)g * kQ8Group + 4 * hl;
			h = vec ? __ldg(reinterpret_cast<const float4 *>(p)) : make_float4(__ldg(p), __ldg(p + 1), __ldg(p + 2), __ldg(p + 3));
		}
		float scale, recip;
		q8_scale(group_absmax_f4(h, lane), scale, recip);
		if (g < groups) {
			sq[g * 16 + hl] = q8_codes4(h, recip);
			if (hl == 0)
				ss[g] = scale;
		}
	}
}

// MODE 0: v7d_q8 (one matrix); 1: v7d_swiglu_q8 (gate, up, SwiGLU epilogue).
// FUSED: the activation arrives as fp32 and is quantised here first.
template <int MODE, bool FUSED>
__global__ void __launch_bounds__(kBlock) k_q8_gemv(GemvArgs p)
{
	using M = F<true>;
	constexpr int NM = MODE == 1 ? 2 : 1;
	extern __shared__ __align__(16) unsigned char smem[];
	const int n = p.n, groups = n / kQ8Group;
	uint32_t *sq = reinterpret_cast<uint32_t *>(smem);
	float *ss = reinterpret_cast<float *>(smem + n);
	const int64_t b = blockIdx.y;
	if (FUSED) {
		stage_quantized(p.xf + b * n, n, sq, ss);
	} else {
		const uint4 *src = reinterpret_cast<const uint4 *>(p.xq + b * n);
		for (int i = threadIdx.x; i < n / 16; i += kBlock)
			reinterpret_cast<uint4 *>(smem)[i] = __ldg(src + i);
		for (int i = threadIdx.x; i < groups; i += kBlock)
			ss[i] = __ldg(p.xs + b * groups + i);
	}
	__syncthreads();
	const int l = threadIdx.x & (kLanes - 1);
	// rows past d compute nothing but stay for the lane shuffles
	const int64_t row_raw = (int64_t)blockIdx.x * kRowsPerBlock + (threadIdx.x >> 3);
	const bool valid = row_raw < p.d;
	const int64_t row = valid ? row_raw : 0;
	const int gend = valid ? groups : 0;
	const uint32_t *w[NM];
	const float *s[NM];
#pragma unroll
	for (int m = 0; m < NM; ++m) {
		w[m] = reinterpret_cast<const uint32_t *>(p.wq[m] + row * n) + l;
		s[m] = p.ws[m] + row * groups;
	}
	float acc[NM];
#pragma unroll
	for (int m = 0; m < NM; ++m)
		acc[m] = 0.0f;
	for (int g0 = 0; g0 < gend; g0 += kUnroll) {
		uint32_t lo[NM][kUnroll], hi[NM][kUnroll];
		float sc[NM][kUnroll];
#pragma unroll
		for (int u = 0; u < kUnroll; ++u)
			if (g0 + u < gend) {
#pragma unroll
				for (int m = 0; m < NM; ++m) {
					lo[m][u] = __ldcs(w[m] + (g0 + u) * 16);
					hi[m][u] = __ldcs(w[m] + (g0 + u) * 16 + 8);
					sc[m][u] = __ldg(s[m] + g0 + u);
				}
			}
#pragma unroll
		for (int u = 0; u < kUnroll; ++u)
			if (g0 + u < gend) {
				const int g = g0 + u;
				const uint32_t a_lo = sq[g * 16 + l], a_hi = sq[g * 16 + 8 + l];
				const float xsg = ss[g];
#pragma unroll
				for (int m = 0; m < NM; ++m) {
					const int dot = lane_dot(a_lo, lo[m][u], a_hi, hi[m][u]);
					acc[m] = M::fma((float)dot, M::mul(sc[m][u], xsg), acc[m]);
				}
			}
	}
	float r[NM];
#pragma unroll
	for (int m = 0; m < NM; ++m)
		r[m] = hadd_lanes(acc[m]);
	if (l == 0 && valid)
		p.out[b * p.d + row] = MODE == 1 ? v7_swiglu(r[0], r[1]) : r[0];
}

// fp32 activation x Q8 weights, SwiGLU epilogue (v7d_swiglu, dual-row path):
// thread l of a row owns lane l, i.e. elements e = l (mod 8).
__global__ void __launch_bounds__(kBlock) k_f32q8_swiglu_gemv(GemvArgs p)
{
	using M = F<true>;
	const int n = p.n, groups = n / kQ8Group;
	const int64_t b = blockIdx.y;
	const int l = threadIdx.x & (kLanes - 1);
	const int64_t row_raw = (int64_t)blockIdx.x * kRowsPerBlock + (threadIdx.x >> 3);
	const bool valid = row_raw < p.d;
	const int64_t row = valid ? row_raw : 0;
	const int gend = valid ? groups : 0;
	const float *x = p.xf + b * n + l;
	const int8_t *w[2] = {p.wq[0] + row * n + l, p.wq[1] + row * n + l};
	const float *s[2] = {p.ws[0] + row * groups, p.ws[1] + row * groups};
	float acc[2] = {0.0f, 0.0f};
	for (int g = 0; g < gend; ++g) {
		int8_t wb[2][8];
		float xv[8];
#pragma unroll
		for (int k = 0; k < 8; ++k) {
			wb[0][k] = __ldcs(w[0] + g * kQ8Group + 8 * k);
			wb[1][k] = __ldcs(w[1] + g * kQ8Group + 8 * k);
			xv[k] = __ldg(x + g * kQ8Group + 8 * k);
		}
		const float sg[2] = {__ldg(s[0] + g), __ldg(s[1] + g)};
#pragma unroll
		for (int k = 0; k < 8; ++k)
#pragma unroll
			for (int m = 0; m < 2; ++m)
				acc[m] = M::fma(xv[k], M::mul((float)wb[m][k], sg[m]), acc[m]);
	}
	const float gsum = hadd_lanes(acc[0]), usum = hadd_lanes(acc[1]);
	if (l == 0 && valid)
		p.out[b * p.d + row] = v7_swiglu(gsum, usum);
}

int check_gemv(const char *what, float *out, int64_t batch, int n, int d)
{
	if (batch < 0 || d < 0)
		return set_error(V7G_ERR_ARG, "%s: negative batch or d", what);
	if (n <= 0 || n % kQ8Group != 0 || n > kMaxN)
		return set_error(V7G_ERR_ARG, "%s: n = %d must be a positive multiple of 64, at most %d", what, n, kMaxN);
	if (batch > 65535)
		return set_error(V7G_ERR_ARG, "%s: batch %lld above 65535", what, (long long)batch);
	if (batch > 0 && d > 0 && !out)
		return set_error(V7G_ERR_ARG, "%s: NULL output", what);
	return V7G_OK;
}

template <typename Kernel>
int launch_gemv(Kernel kernel, const char *what, const GemvArgs &a, int64_t batch, size_t smem, void *stream)
{
	DeviceInfo dev;
	int rc = current_device(&dev);
	if (rc != V7G_OK)
		return rc;
	if (smem > 48 * 1024 && cudaFuncSetAttribute((const void *)kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
		return check_launch(what);
	const dim3 grid((unsigned)((a.d + kRowsPerBlock - 1) / kRowsPerBlock), (unsigned)batch);
	kernel<<<grid, kBlock, smem, (cudaStream_t)stream>>>(a);
	return check_launch(what);
}

bool weights_ok(const int8_t *q, const float *s) { return q && s && (reinterpret_cast<uintptr_t>(q) & 3) == 0; }

} // namespace
} // namespace v7g

using namespace v7g;

extern "C" {

int v7g_q8_gemv(float *out, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws, int64_t batch, int n, int d, void *stream)
{
	const char *what = "v7g_q8_gemv";
	int rc = check_gemv(what, out, batch, n, d);
	if (rc != V7G_OK)
		return rc;
	if (batch == 0 || d == 0)
		return clear_error();
	if (!xq || !xs || !aligned16(xq) || !weights_ok(wq, ws))
		return set_error(V7G_ERR_ARG, "%s: NULL pointer, activation codes not 16-byte or weight codes not 4-byte aligned", what);
	GemvArgs a{out, xq, xs, nullptr, {wq, wq}, {ws, ws}, n, d};
	return launch_gemv(k_q8_gemv<0, false>, what, a, batch, (size_t)n + (size_t)n / 16, stream);
}

int v7g_q8_fused_gemv(float *out, const float *x, const int8_t *wq, const float *ws, int64_t batch, int n, int d, void *stream)
{
	const char *what = "v7g_q8_fused_gemv";
	int rc = check_gemv(what, out, batch, n, d);
	if (rc != V7G_OK)
		return rc;
	if (batch == 0 || d == 0)
		return clear_error();
	if (!x || !weights_ok(wq, ws))
		return set_error(V7G_ERR_ARG, "%s: NULL pointer or weight codes not 4-byte aligned", what);
	GemvArgs a{out, nullptr, nullptr, x, {wq, wq}, {ws, ws}, n, d};
	return launch_gemv(k_q8_gemv<0, true>, what, a, batch, (size_t)n + (size_t)n / 16, stream);
}

int v7g_swiglu_q8_gemv(float *out, const int8_t *xq, const float *xs, const int8_t *gate_q, const float *gate_s, const int8_t *up_q, const float *up_s, int64_t batch, int n, int d, void *stream)
{
	const char *what = "v7g_swiglu_q8_gemv";
	int rc = check_gemv(what, out, batch, n, d);
	if (rc != V7G_OK)
		return rc;
	if (batch == 0 || d == 0)
		return clear_error();
	if (!xq || !xs || !aligned16(xq) || !weights_ok(gate_q, gate_s) || !weights_ok(up_q, up_s))
		return set_error(V7G_ERR_ARG, "%s: NULL pointer, activation codes not 16-byte or weight codes not 4-byte aligned", what);
	GemvArgs a{out, xq, xs, nullptr, {gate_q, up_q}, {gate_s, up_s}, n, d};
	return launch_gemv(k_q8_gemv<1, false>, what, a, batch, (size_t)n + (size_t)n / 16, stream);
}

int v7g_swiglu_f32q8_gemv(float *out, const float *x, const int8_t *gate_q, const float *gate_s, const int8_t *up_q, const float *up_s, int64_t batch, int n, int d, void *stream)
{
	const char *what = "v7g_swiglu_f32q8_gemv";
	int rc = check_gemv(what, out, batch, n, d);
	if (rc != V7G_OK)
		return rc;
	if (batch == 0 || d == 0)
		return clear_error();
	if (!x || !gate_q || !gate_s || !up_q || !up_s)
		return set_error(V7G_ERR_ARG, "%s: NULL pointer", what);
	GemvArgs a{out, nullptr, nullptr, x, {gate_q, up_q}, {gate_s, up_s}, n, d};
	return launch_gemv(k_f32q8_swiglu_gemv, what, a, batch, 0, stream);
}

} // extern "C"
