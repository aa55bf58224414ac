/* v7_oracle.c -- CPU restatement of v7's elementwise / reduction kernels.
 *
 * TEST INFRASTRUCTURE ONLY (see v7_oracle.h): the parity checker for the
 * sm_100a kernels, never a product code path.
 *
 * Written in plain C, scalar, with the reference's 8-lane YMM registers
 * spelled out as float[8] arrays so the order of every rounding step is
 * visible.  Build with -ffp-contract=off: a multiply followed by an add is two
 * roundings unless fmaf() is written, exactly as in the reference where only
 * vfmadd* fuse.  MXCSR FTZ+DAZ is switched on around the kernels the
 * reference runs on its dispatched worker threads, so denormals behave as
 * there.
 */
#include "v7_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <immintrin.h>
#include <xmmintrin.h>

/* ------------------------------------------------------------------------ */
/* x86 scalar semantics used by the reference                                */
/* ------------------------------------------------------------------------ */

/* MAXPS/MAXSS dst = max(a, b): returns b when either is NaN or both are zero. */
static inline float x86_max(float a, float b) { return a > b ? a : b; }
/* MINPS/MINSS dst = min(a, b): returns b when either is NaN or both are zero. */
static inline float x86_min(float a, float b) { return a < b ? a : b; }

/* CVTPS2DQ under round-to-nearest-even: NaN and out-of-range give INT_MIN. */
static inline int32_t x86_cvtps2dq(float p)
{
	if (!(fabsf(p) < 2147483648.0f))
		return INT32_MIN;
	return (int32_t)rintf(p);
}

/* VPACKSSDW -> VPACKSSWB -> VPMAXSB(-127): int32 to int8 with saturation,
   then the -128 code lifted to -127 (quantize_kernel.inc:100-103). */
static inline int8_t x86_pack_q8(int32_t v)
{
	if (v > 32767)
		v = 32767;
	if (v < -32768)
		v = -32768;
	if (v > 127)
		v = 127;
	if (v < -128)
		v = -128;
	if (v < -127)
		v = -127;
	return (int8_t)v;
}

static inline float bits_to_float(uint32_t u)
{
	float f;
	memcpy(&f, &u, 4);
	return f;
}

#define MXCSR_FTZ_DAZ 0x8040u

/* ------------------------------------------------------------------------ */
/* shared pieces                                                             */
/* ------------------------------------------------------------------------ */

/* HADD_YMM (v7_macros.inc:38-45): low128 + high128, then (e0+e1) + (e2+e3). */
static inline float hadd8(const float s[8])
{
	float t0 = s[0] + s[4], t1 = s[1] + s[5], t2 = s[2] + s[6], t3 = s[3] + s[7];
	float u0 = t0 + t1, u1 = t2 + t3;
	return u0 + u1;
}

/* (A+B)+(C+D) merge of the four accumulators (rmsnorm_kernel.inc:43-45),
   then HADD_YMM. */
static inline float merge4x8(float acc[4][8])
{
	float s[8];
	for (int c = 0; c < 8; ++c) {
		float ab = acc[0][c] + acc[1][c];
		float cd = acc[2][c] + acc[3][c];
		s[c] = ab + cd;
	}
	return hadd8(s);
}

/* Sum of squares, 8-float block b feeding accumulator b % 4 with FMA
   (rmsnorm_kernel.inc:22-40; RMSNORM_ROPE_BODY v7_macros.inc:266-289;
   rmsnorm_quantize_kernel.inc Phase 1).  n % 32 == 0. */
static float sumsq_blocks(const float *x, int n)
{
	float acc[4][8];
	memset(acc, 0, sizeof(acc));
	int blocks = n / 8;
	for (int b = 0; b < blocks; ++b)
		for (int c = 0; c < 8; ++c) {
			float v = x[8 * b + c];
			acc[b & 3][c] = fmaf(v, v, acc[b & 3][c]);
		}
	return merge4x8(acc);
}

/* COMPUTE_RMS_SCALE (v7_macros.inc:348-354): four exact IEEE operations. */
static inline float rms_scale(float ss, float nf, float eps)
{
	float mean = ss / nf;
	float val = mean + eps;
	float r = sqrtf(val);
	return 1.0f / r;
}

/* EVAL_SIGMOID (v7_macros.inc:98-160), constants from math_data.inc:16-34
   and sampler.inc:75.  Runs under the caller's MXCSR. */
static const uint32_t SIG_C5 = 0x3AADD303u, SIG_C4 = 0x3C1E7411u, SIG_C3 = 0x3D635B9Bu, SIG_C2 = 0x3E75FCE0u, SIG_C1 = 0x3F317215u;
static inline float sigmoid_v7(float g)
{
	float t = -g;                      /* sign flip (vxorps with the sign mask) */
	t = x86_max(t, -80.0f);            /* vmaxps t, t, -80 */
	t = x86_min(t, 80.0f);             /* vminps t, t, 80 */
	float fx = t * 1.4426950408889634f; /* x * log2(e) */
	float ip = rintf(fx);              /* vroundps mode 0 */
	float f = fx - ip;
	int32_t ipi = (int32_t)ip;         /* vcvttps2dq of an integral value */
	float p = fmaf(bits_to_float(SIG_C5), f, bits_to_float(SIG_C4));
	p = fmaf(p, f, bits_to_float(SIG_C3));
	p = fmaf(p, f, bits_to_float(SIG_C2));
	p = fmaf(p, f, bits_to_float(SIG_C1));
	p = fmaf(p, f, 1.0f);
	float two_ip = bits_to_float((uint32_t)(ipi + 127) << 23);
	float e = two_ip * p;
	float d = e + 1.0f;
	return 1.0f / d;
}

/* SwiGLU product order (sig * g) * u (swiglu_q8_kernel.inc:204-209). */
static inline float swiglu_v7(float g, float u)
{
	float sg = sigmoid_v7(g) * g;
	return sg * u;
}

/* One full group of 64 values: absmax tree, scale, codes
   (quantize_kernel.inc:62-106). */
static void quantize_group64(int8_t *q, float *s, const float *x)
{
	float a[64];
	for (int i = 0; i < 64; ++i)
		a[i] = fabsf(x[i]);
	float m[8];
	for (int c = 0; c < 8; ++c) {
		float m01 = x86_max(a[c], a[8 + c]);
		float m23 = x86_max(a[16 + c], a[24 + c]);
		float m03 = x86_max(m01, m23);
		float m45 = x86_max(a[32 + c], a[40 + c]);
		float m67 = x86_max(a[48 + c], a[56 + c]);
		float m47 = x86_max(m45, m67);
		m[c] = x86_max(m03, m47);
	}
	float v[4];
	for (int j = 0; j < 4; ++j)
		v[j] = x86_max(m[j], m[j + 4]);
	float w0 = x86_max(v[0], v[2]);
	float w1 = x86_max(v[1], v[3]);
	float wmax = x86_max(w0, w1);
	wmax = x86_max(wmax, ORC_Q8_WMAX_FLOOR);
	float scale = wmax / 127.0f;
	*s = scale;
	float recip = 1.0f / scale;
	for (int i = 0; i < 64; ++i)
		q[i] = x86_pack_q8(x86_cvtps2dq(x[i] * recip));
}

/* A trailing group of r < 64 values: scalar path (quantize_kernel.inc:119-152). */
static void quantize_tail(int8_t *q, float *s, const float *x, int r)
{
	float wmax = 0.0f;
	for (int i = 0; i < r; ++i)
		wmax = x86_max(fabsf(x[i]), wmax);
	wmax = x86_max(wmax, ORC_Q8_WMAX_FLOOR);
	float scale = wmax / 127.0f;
	*s = scale;
	float recip = 1.0f / scale;
	for (int i = 0; i < r; ++i) {
		float p = x[i] * recip;
		p = x86_max(p, -127.0f);
		p = x86_min(p, 127.0f);
		q[i] = (int8_t)(int32_t)rintf(p);
	}
}

static void quantize_vec(int8_t *q, float *s, const float *x, int n)
{
	int g = 0;
	for (; (g + 1) * ORC_Q8_GS <= n; ++g)
		quantize_group64(q + (int64_t)g * ORC_Q8_GS, s + g, x + (int64_t)g * ORC_Q8_GS);
	int r = n - g * ORC_Q8_GS;
	if (r > 0)
		quantize_tail(q + (int64_t)g * ORC_Q8_GS, s + g, x + (int64_t)g * ORC_Q8_GS, r);
}

/* ------------------------------------------------------------------------ */
/* row workers                                                               */
/* ------------------------------------------------------------------------ */

static void rmsnorm_row(float *o, const float *x, const float *w, int n, float eps)
{
	float scale = rms_scale(sumsq_blocks(x, n), (float)n, eps);
	for (int i = 0; i < n; ++i) {
		float t = x[i] * scale;
		o[i] = t * w[i];
	}
}

static void fused_add_rmsnorm_row(float *o, float *r, const float *a, const float *w, int n, float eps)
{
	float acc[4][8];
	memset(acc, 0, sizeof(acc));
	int blocks = n / 8;
	int left = blocks & 3;
	/* leftover blocks first, all into accumulator A */
	for (int b = 0; b < left; ++b)
		for (int c = 0; c < 8; ++c) {
			float sv = r[8 * b + c] + a[8 * b + c];
			r[8 * b + c] = sv;
			acc[0][c] = fmaf(sv, sv, acc[0][c]);
		}
	for (int b = left; b < blocks; ++b)
		for (int c = 0; c < 8; ++c) {
			float sv = r[8 * b + c] + a[8 * b + c];
			r[8 * b + c] = sv;
			acc[(b - left) & 3][c] = fmaf(sv, sv, acc[(b - left) & 3][c]);
		}
	float scale = rms_scale(merge4x8(acc), (float)n, eps);
	for (int i = 0; i < n; ++i) {
		float t = r[i] * scale;
		o[i] = t * w[i];
	}
}

/* RMSNORM_ROPE_BODY (v7_macros.inc:263-339) for one head. */
static void rmsnorm_rope_head(float *x, int head_dim, const float *w, const float *cs, const float *sn, int64_t pos, float eps)
{
	float scale = rms_scale(sumsq_blocks(x, head_dim), (float)head_dim, eps);
	if (pos == 0) {
		for (int i = 0; i < head_dim; ++i) {
			float t = x[i] * scale;
			x[i] = t * w[i];
		}
		return;
	}
	int half = head_dim / 2;
	for (int j = 0; j < half; ++j) {
		float e = (x[j] * scale) * w[j];
		float o = (x[j + half] * scale) * w[j + half];
		float ec = e * cs[j];
		float es = e * sn[j];
		x[j] = fmaf(-o, sn[j], ec);
		x[j + half] = fmaf(o, cs[j], es);
	}
}

/* RoPE without the norm, one head in place (rope_only_kernel.inc:13-50):
   position 0 is the identity and writes nothing; otherwise each pair (j,
   j + half) becomes (lo*cos - hi*sin, lo*sin + hi*cos) with the product by
   cos / sin of lo rounded and the hi term fused (vfnmadd231ps /
   vfmadd231ps). */
static void rope_only_head(float *x, int head_dim, const float *cs, const float *sn, int64_t pos)
{
	if (pos == 0)
		return;
	int half = head_dim / 2;
	for (int j = 0; j < half; ++j) {
		float lo = x[j], hi = x[j + half];
		float lc = lo * cs[j];
		float ls = lo * sn[j];
		x[j] = fmaf(-hi, sn[j], lc);
		x[j + half] = fmaf(hi, cs[j], ls);
	}
}

static void rmsnorm_quantize_row(int8_t *q, float *s, const float *x, const float *w, int n, float eps)
{
	float scale = rms_scale(sumsq_blocks(x, n), (float)n, eps);
	float norm[ORC_Q8_GS];
	for (int g = 0; g < n / ORC_Q8_GS; ++g) {
		const float *xg = x + g * ORC_Q8_GS;
		const float *wg = w + g * ORC_Q8_GS;
		for (int i = 0; i < ORC_Q8_GS; ++i) {
			float t = scale * xg[i];
			norm[i] = t * wg[i];
		}
		quantize_group64(q + g * ORC_Q8_GS, s + g, norm);
	}
}

/* ------------------------------------------------------------------------ */
/* RoPE tables: the x87 extended-precision producer                         */
/* ------------------------------------------------------------------------ */

/* The reference builds its tables with x87 instructions at extended
   precision, round to nearest, all exceptions masked (control word 0x037F,
   fused_f32_kernel.inc:22,117-118), keeping some intermediates in 80-bit
   registers and storing others as doubles.  long double on x86-64 is that
   80-bit format and its arithmetic compiles to the same x87 operations; the
   instructions C has no operator for are issued directly. */
#define X87_CW_EXTENDED_NEAREST 0x037F

static unsigned short x87_set_cw(unsigned short cw)
{
	unsigned short old;
	__asm__ __volatile__("fnstcw %0" : "=m"(old));
	__asm__ __volatile__("fldcw %0" : : "m"(cw));
	return old;
}

/* y * log2(x) */
static long double x87_fyl2x(long double x, long double y)
{
	long double r;
	__asm__("fyl2x" : "=t"(r) : "0"(x), "u"(y) : "st(1)");
	return r;
}

static long double x87_frndint(long double x)
{
	long double r;
	__asm__("frndint" : "=t"(r) : "0"(x));
	return r;
}

/* 2^x - 1 for |x| <= 1 */
static long double x87_f2xm1(long double x)
{
	long double r;
	__asm__("f2xm1" : "=t"(r) : "0"(x));
	return r;
}

/* x * 2^trunc(n) */
static long double x87_fscale(long double x, long double n)
{
	long double r;
	__asm__("fscale" : "=t"(r) : "0"(x), "u"(n));
	return r;
}

static void x87_fsincos(long double a, long double *c, long double *s)
{
	long double cr, sr;
	__asm__("fsincos" : "=t"(cr), "=u"(sr) : "0"(a));
	*c = cr;
	*s = sr;
}

/* base^(-j/half) at extended precision: -j/half, times log2(base) by fyl2x,
   split into integer and fraction, 2^fraction by f2xm1 + 1, scaled by the
   integer power (RBIT_CALC_INV_FREQ, fused_f32_kernel.inc:120-137). */
static long double inv_freq_x87(float base, int j, int half)
{
	long double e = (long double)j / (long double)half;
	long double y = x87_fyl2x((long double)base, -e);
	long double ip = x87_frndint(y);
	long double p = x87_f2xm1(y - ip) + 1.0L;
	return x87_fscale(p, ip);
}

/* 2*pi as the double the reference stores (fused_f32_kernel.inc:65-66) */
static const double kTwoPi = 6.28318530717958647692;

/* llama3 frequency scaling for one j (fused_f32_kernel.inc:186-256): the
   values the reference keeps in double slots are rounded to double at the
   same points, the rest stays at extended precision. */
static double llama3_freq_x87(float base, int j, int half, double factor, double high, double low, double old_ctx, double low_wl, double high_wl)
{
	long double inv80 = inv_freq_x87(base, j, half);
	double inv = (double)inv80;
	double wavelen = (double)((long double)kTwoPi / inv80);
	double ifl = low_wl < wavelen ? (double)((long double)inv / (long double)factor) : inv;
	long double num = (long double)old_ctx / (long double)wavelen - (long double)low;
	long double den = (long double)high - (long double)low;
	double smooth = (double)(num / den);
	long double t1 = (1.0L - (long double)smooth) * ((long double)ifl / (long double)factor);
	long double t2 = (long double)smooth * (long double)ifl;
	double smoothed = (double)(t1 + t2);
	int medium = (high_wl < wavelen && low_wl >= wavelen) || high_wl == wavelen;
	return medium ? smoothed : ifl;
}

int orc_rope_freqs(double *freqs, int half, float base, int scaling, float factor, float high_freq_factor, float low_freq_factor, int orig_max_pos)
{
	if (!freqs || half <= 0 || half > ORC_ROPE_MAX_HALF || (scaling != 0 && scaling != 1))
		return -1;
	unsigned short saved = x87_set_cw(X87_CW_EXTENDED_NEAREST);
	if (scaling == 0) {
		for (int j = 0; j < half; ++j)
			freqs[j] = (double)inv_freq_x87(base, j, half);
	} else {
		double f = factor, hi = high_freq_factor, lo = low_freq_factor, old = (double)orig_max_pos;
		double low_wl = (double)((long double)old / (long double)lo);
		double high_wl = (double)((long double)old / (long double)hi);
		for (int j = 0; j < half; ++j)
			freqs[j] = llama3_freq_x87(base, j, half, f, hi, lo, old, low_wl, high_wl);
	}
	x87_set_cw(saved);
	return 0;
}

/* One table row: angle = freq_j * pos at extended precision, fsincos, each
   stored as fp32 (fused_f32_kernel.inc:262-283).  Columns half..stride-1 are
   zero. */
static void rope_table_row(float *cs, float *sn, int64_t pos, int half, int stride, const double *freqs)
{
	unsigned short saved = x87_set_cw(X87_CW_EXTENDED_NEAREST);
	double pd = (double)pos;
	for (int j = 0; j < half; ++j) {
		long double c, s;
		x87_fsincos((long double)freqs[j] * (long double)pd, &c, &s);
		cs[j] = (float)c;
		sn[j] = (float)s;
	}
	for (int j = half; j < stride; ++j)
		cs[j] = sn[j] = 0.0f;
	x87_set_cw(saved);
}

/* ------------------------------------------------------------------------ */
/* Q8-weight GEMVs                                                          */
/* ------------------------------------------------------------------------ */

/* One activation byte times one weight byte the way vpsignb + vpmaddubsw
   form it (q8_kernel.inc:22-36, swiglu_q8_kernel.inc:16-33): the weight takes
   the activation's sign (negated in 8 bits, so -128 stays -128; zero when the
   activation is zero), times the activation's magnitude as an unsigned byte
   (|-128| = 128).  Equal to a * w for every weight in [-127, 127], the
   exporter's contract; no pair sum reaches the int16 saturation bound. */
static inline int32_t x86_signmul(int8_t a, int8_t w)
{
	int32_t ua = a < 0 ? -(int32_t)a : (int32_t)a;
	int8_t sw = a < 0 ? (int8_t)(uint8_t)(0u - (uint8_t)w) : (a == 0 ? 0 : w);
	return ua * (int32_t)sw;
}

/* The 8 int32 lane dots of one 64-byte group: lane l sums bytes 4l..4l+3 of
   the low 32 bytes and 4l..4l+3 of the high 32 (vpmaddwd pair-adds, then
   vpaddd low + high). */
static inline void q8_lane_dots(int32_t dot[8], const int8_t *a, const int8_t *w)
{
	for (int l = 0; l < 8; ++l) {
		int32_t s = 0;
		for (int k = 0; k < 4; ++k)
			s += x86_signmul(a[4 * l + k], w[4 * l + k]) + x86_signmul(a[32 + 4 * l + k], w[32 + 4 * l + k]);
		dot[l] = s;
	}
}

/* Q8 x Q8 dot of one weight row with the activation: per group the lane dots
   converted to float (exact), the weight scale times the activation scale
   (rounded), one FMA per lane into 8 lane accumulators; HADD_YMM at the end
   (q8_kernel.inc:141-162, 176-201). */
static float q8_row_dot(const int8_t *xq, const float *xs, const int8_t *wq, const float *ws, int n)
{
	float acc[8] = { 0 };
	int32_t dot[8];
	for (int g = 0; g < n / ORC_Q8_GS; ++g) {
		q8_lane_dots(dot, xq + (int64_t)g * ORC_Q8_GS, wq + (int64_t)g * ORC_Q8_GS);
		float cs = ws[g] * xs[g];
		for (int l = 0; l < 8; ++l)
			acc[l] = fmaf((float)dot[l], cs, acc[l]);
	}
	return hadd8(acc);
}

/* fp32 activation x Q8 weight row, the dual-row arithmetic of
   swiglu_kernel.inc:30-47,138-249: weight to float times the group scale
   (rounded), one FMA per element into lane e % 8 of a single accumulator. */
static float f32q8_row_dot_dual(const float *x, const int8_t *wq, const float *ws, int n)
{
	float acc[8] = { 0 };
	for (int e = 0; e < n; ++e) {
		float wf = (float)wq[e] * ws[e / ORC_Q8_GS];
		acc[e % 8] = fmaf(x[e], wf, acc[e % 8]);
	}
	return hadd8(acc);
}

/* The same for the single-row path (the last row of an odd-sized work
   chunk, swiglu_kernel.inc:253-375): four accumulators, 8-element block b
   feeding accumulator b % 4 through the 256-element loop and the 64/32/16
   tails, every later 8-element tail block accumulator 0; merged
   (acc0 + acc1) + (acc2 + acc3) before HADD_YMM. */
static float f32q8_row_dot_single(const float *x, const int8_t *wq, const float *ws, int n)
{
	float acc[4][8] = { { 0 } };
	const int n256 = n / 256 * 256;
	for (int e = 0; e < n; ++e) {
		int a = e < n256 + 112 ? (e / 8) % 4 : 0;
		float wf = (float)wq[e] * ws[e / ORC_Q8_GS];
		acc[a][e % 8] = fmaf(x[e], wf, acc[a][e % 8]);
	}
	float s[8];
	for (int l = 0; l < 8; ++l)
		s[l] = (acc[0][l] + acc[1][l]) + (acc[2][l] + acc[3][l]);
	return hadd8(s);
}


/* ------------------------------------------------------------------------ */
/* SwiGLU -> Q8 in AVX2, the reference's own instruction forms               */
/* ------------------------------------------------------------------------ */

/* The same operations as swiglu_v7 and quantize_group64 above, eight lanes
 * per instruction the way the reference's AVX2 kernels run them
 * (EVAL_SIGMOID v7_macros.inc:98-160: vxorps, vmaxps, vminps, vmulps,
 * vroundps, vsubps, vcvttps2dq, vfmadd, vpaddd/vpslld, vmulps, vaddps,
 * vdivps; quantize_kernel.inc:62-106: vandps, the vmaxps tree, vdivss,
 * vmulps, vcvtps2dq, vpackssdw, vpacksswb, vpmaxsb).  The scalar versions
 * are the readable statement and this one the fast one: the CPU baseline
 * times it, and tests/test_oracle_props.py checks the two give identical
 * bits (NaN, infinities and subnormals included).  Runs under the job's
 * MXCSR (FTZ+DAZ, as the reference's dispatched workers). */
static inline __m256 sigmoid8_v7(__m256 g)
{
	const __m256 sign = _mm256_castsi256_ps(_mm256_set1_epi32((int)0x80000000u));
	__m256 t = _mm256_xor_ps(g, sign);
	t = _mm256_max_ps(t, _mm256_set1_ps(-80.0f)); /* NaN -> -80, as x86_max(t, -80) */
	t = _mm256_min_ps(t, _mm256_set1_ps(80.0f));
	const __m256 fx = _mm256_mul_ps(t, _mm256_set1_ps(1.4426950408889634f));
	const __m256 ip = _mm256_round_ps(fx, _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
	const __m256 f = _mm256_sub_ps(fx, ip);
	const __m256i ipi = _mm256_cvttps_epi32(ip);
	__m256 p = _mm256_fmadd_ps(_mm256_set1_ps(bits_to_float(SIG_C5)), f, _mm256_set1_ps(bits_to_float(SIG_C4)));
	p = _mm256_fmadd_ps(p, f, _mm256_set1_ps(bits_to_float(SIG_C3)));
	p = _mm256_fmadd_ps(p, f, _mm256_set1_ps(bits_to_float(SIG_C2)));
	p = _mm256_fmadd_ps(p, f, _mm256_set1_ps(bits_to_float(SIG_C1)));
	p = _mm256_fmadd_ps(p, f, _mm256_set1_ps(1.0f));
	const __m256 two = _mm256_castsi256_ps(_mm256_slli_epi32(_mm256_add_epi32(ipi, _mm256_set1_epi32(127)), 23));
	const __m256 d = _mm256_add_ps(_mm256_mul_ps(two, p), _mm256_set1_ps(1.0f));
	return _mm256_div_ps(_mm256_set1_ps(1.0f), d);
}

/* One row of SwiGLU -> Q8 (n % 64 == 0): h = (sig(g) * g) * u per 64-group,
 * then the group's scale and codes. */
static void swiglu_q8_row_avx2(int8_t *q, float *s, const float *g, const float *u, int n)
{
	const __m256 absmask = _mm256_castsi256_ps(_mm256_set1_epi32(0x7fffffff));
	const __m256i order = _mm256_setr_epi32(0, 4, 1, 5, 2, 6, 3, 7);
	const __m256i floor127 = _mm256_set1_epi8(-127);
	for (int grp = 0; grp < n / ORC_Q8_GS; ++grp) {
		const float *gg = g + (int64_t)grp * ORC_Q8_GS, *uu = u + (int64_t)grp * ORC_Q8_GS;
		__m256 h[8], a[8];
		for (int b = 0; b < 8; ++b) {
			const __m256 gv = _mm256_loadu_ps(gg + 8 * b);
			h[b] = _mm256_mul_ps(_mm256_mul_ps(sigmoid8_v7(gv), gv), _mm256_loadu_ps(uu + 8 * b));
			a[b] = _mm256_and_ps(h[b], absmask);
		}
		/* the MAXPS tree: blocks (0,1),(2,3) -> (01,23), (4,5),(6,7) -> (45,67), then (03,47) */
		const __m256 m03 = _mm256_max_ps(_mm256_max_ps(a[0], a[1]), _mm256_max_ps(a[2], a[3]));
		const __m256 m47 = _mm256_max_ps(_mm256_max_ps(a[4], a[5]), _mm256_max_ps(a[6], a[7]));
		const __m256 m = _mm256_max_ps(m03, m47);
		/* lanes j vs j + 4, then (0,2), (1,3), then (0,1) */
		const __m128 v = _mm_max_ps(_mm256_castps256_ps128(m), _mm256_extractf128_ps(m, 1));
		const __m128 w = _mm_max_ps(v, _mm_movehl_ps(v, v));
		__m128 wmax = _mm_max_ss(w, _mm_shuffle_ps(w, w, 1));
		wmax = _mm_max_ss(wmax, _mm_set_ss(ORC_Q8_WMAX_FLOOR));
		const __m128 scale = _mm_div_ss(wmax, _mm_set_ss(127.0f));
		const __m128 recip = _mm_div_ss(_mm_set_ss(1.0f), scale);
		s[grp] = _mm_cvtss_f32(scale);
		const __m256 r8 = _mm256_broadcastss_ps(recip);
		__m256i c[8];
		for (int b = 0; b < 8; ++b)
			c[b] = _mm256_cvtps_epi32(_mm256_mul_ps(h[b], r8));
		for (int half = 0; half < 2; ++half) {
			const __m256i p01 = _mm256_packs_epi32(c[4 * half], c[4 * half + 1]);
			const __m256i p23 = _mm256_packs_epi32(c[4 * half + 2], c[4 * half + 3]);
			__m256i bytes = _mm256_packs_epi16(p01, p23);
			bytes = _mm256_permutevar8x32_epi32(bytes, order);
			bytes = _mm256_max_epi8(bytes, floor127);
			_mm256_storeu_si256((__m256i *)(q + (int64_t)grp * ORC_Q8_GS + 32 * half), bytes);
		}
	}
}

/* ------------------------------------------------------------------------ */
/* synthetic inputs: the library's counter-based N(mean, std) generator       */
/* ------------------------------------------------------------------------ */

/* A restatement of v7g_fill_normal (v7multiplikator_b200/csrc/add.cu,
 * k_fill_normal, fill_ln, fill_cos2pi) -- not reference code: the generator of
 * the bench's synthetic inputs, restated so that the CPU legs of the bench and
 * the multi-GPU verification see the same input bytes as the GPU without
 * copying them from a device.  Box-Muller from correctly rounded IEEE
 * operations in the same order as the device code (fmaf where it fuses, one
 * rounding per * + / otherwise; this file is built with -ffp-contract=off),
 * so the values agree bit for bit. */
static inline uint64_t fill_mix64(uint64_t z)
{
	z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
	z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
	return z ^ (z >> 31);
}

static inline float f_bits(uint32_t b)
{
	float f;
	memcpy(&f, &b, 4);
	return f;
}

static inline uint32_t bits_f(float f)
{
	uint32_t b;
	memcpy(&b, &f, 4);
	return b;
}

/* ln u for u in [2^-24, 1]: u = 2^e m, m in [sqrt(1/2), sqrt(2)), ln m = 2 atanh(s) */
static float fill_ln(float u)
{
	uint32_t b = bits_f(u);
	int e = (int)(b >> 23) - 127;
	b = (b & 0x007fffffu) | 0x3f800000u;
	if (b > 0x3FB504F3u) {
		b -= 0x00800000u;
		e += 1;
	}
	const float m = f_bits(b);
	const float s = (m - 1.0f) / (m + 1.0f);
	const float x = s * s;
	float p = fmaf(x, f_bits(0x3E3A2E8Cu), f_bits(0x3E638E39u));
	p = fmaf(x, p, f_bits(0x3E924925u));
	p = fmaf(x, p, f_bits(0x3ECCCCCDu));
	p = fmaf(x, p, f_bits(0x3F2AAAABu));
	p = fmaf(x, p, 2.0f);
	return fmaf((float)e, f_bits(0x3F317218u), s * p);
}

/* cos(2 pi v) for v in [0, 1): quadrant and Taylor series of cos / sin (f pi/2) */
static float fill_cos2pi(float v)
{
	const float v4 = v * 4.0f;
	const int q = (int)v4;
	const float f = v4 - (float)q;
	const float x = f * f;
	float c = fmaf(x, f_bits(0xB1DB7128u), f_bits(0x34FCE9C5u));
	c = fmaf(x, c, f_bits(0xB7D368F9u));
	c = fmaf(x, c, f_bits(0x3A70FA83u));
	c = fmaf(x, c, f_bits(0xBCAAE9E4u));
	c = fmaf(x, c, f_bits(0x3E81E0F8u));
	c = fmaf(x, c, f_bits(0xBF9DE9E6u));
	c = fmaf(x, c, 1.0f);
	float sn = fmaf(x, f_bits(0x33747A1Au), f_bits(0xB67183A8u));
	sn = fmaf(x, sn, f_bits(0x39283C1Au));
	sn = fmaf(x, sn, f_bits(0xBB996966u));
	sn = fmaf(x, sn, f_bits(0x3DA335E3u));
	sn = fmaf(x, sn, f_bits(0xBF255DE7u));
	sn = fmaf(x, sn, f_bits(0x3FC90FDBu));
	sn = f * sn;
	return q == 0 ? c : q == 1 ? -sn : q == 2 ? -c : sn;
}

static void fill_normal_row(float *dst, int64_t row, int64_t n, uint64_t seed, float mean, float std)
{
	const uint64_t key = fill_mix64(seed ^ 0x9e3779b97f4a7c15ull);
	for (int64_t c = 0; c < n; ++c) {
		const uint64_t h = fill_mix64(key ^ fill_mix64((uint64_t)row * 0xd1b54a32d192ed03ull + (uint64_t)c));
		const float u1 = ((float)(uint32_t)(h >> 40) + 1.0f) * 5.96046448e-08f;
		const float u2 = (float)(uint32_t)(h & 0xffffffu) * 5.96046448e-08f;
		const float z = sqrtf(-2.0f * fill_ln(u1)) * fill_cos2pi(u2);
		dst[c] = mean + std * z;
	}
}

/* ------------------------------------------------------------------------ */
/* row-parallel driver                                                       */
/* ------------------------------------------------------------------------ */

typedef struct job {
	int kind;
	int64_t r0, r1;
	int ftz;
	/* arguments */
	float *fo;
	float *fr;
	const float *fx;
	const float *fy;
	const float *fw;
	const float *fc;
	const float *fs;
	int8_t *q;
	float *sc;
	int64_t n64;
	int n, heads, rope_max_dim;
	int64_t pos0;
	float eps;
	const double *freqs;
	/* GEMV: activation codes / scales (or fp32 activations in fx), weight
	   matrices 1 (gate or the only one) and 2 (up) */
	const int8_t *qin;
	const float *sin_;
	const int8_t *qw1, *qw2;
	const float *sw1, *sw2;
	int d, variant;
	/* synthetic fill */
	uint64_t seed;
	float mean, std;
} job;

enum { K_RMSNORM, K_ADD_RMSNORM, K_ROPE, K_SWIGLU, K_QUANT, K_SWIGLU_Q8, K_ADD, K_RMSNORM_Q8, K_ROPE_ONLY, K_ROPE_TABLE,
       K_Q8_GEMV, K_SWIGLU_Q8_GEMV, K_SWIGLU_F32Q8_GEMV, K_Q8_FUSED_GEMV, K_FILL_NORMAL, K_SWIGLU_Q8_AVX2 };

static void gemv_row(const job *j, int64_t r)
{
	const int64_t b = r / j->d, i = r % j->d;
	const int n = j->n, ng = n / ORC_Q8_GS;
	const int8_t *w1 = j->qw1 + i * (int64_t)n;
	const float *s1 = j->sw1 + i * (int64_t)ng;
	switch (j->kind) {
	case K_Q8_GEMV:
		j->fo[r] = q8_row_dot(j->qin + b * (int64_t)n, j->sin_ + b * (int64_t)ng, w1, s1, n);
		break;
	case K_Q8_FUSED_GEMV: {
		int8_t xq[ORC_GEMV_MAX_N];
		float xs[ORC_GEMV_MAX_N / ORC_Q8_GS];
		quantize_vec(xq, xs, j->fx + b * (int64_t)n, n);
		j->fo[r] = q8_row_dot(xq, xs, w1, s1, n);
		break;
	}
	case K_SWIGLU_Q8_GEMV: {
		const int8_t *xq = j->qin + b * (int64_t)n;
		const float *xs = j->sin_ + b * (int64_t)ng;
		float g = q8_row_dot(xq, xs, w1, s1, n);
		float u = q8_row_dot(xq, xs, j->qw2 + i * (int64_t)n, j->sw2 + i * (int64_t)ng, n);
		j->fo[r] = swiglu_v7(g, u);
		break;
	}
	case K_SWIGLU_F32Q8_GEMV: {
		const float *x = j->fx + b * (int64_t)n;
		float (*dot)(const float *, const int8_t *, const float *, int) = j->variant ? f32q8_row_dot_single : f32q8_row_dot_dual;
		float g = dot(x, w1, s1, n);
		float u = dot(x, j->qw2 + i * (int64_t)n, j->sw2 + i * (int64_t)ng, n);
		j->fo[r] = swiglu_v7(g, u);
		break;
	}
	}
}

static void run_job(job *j)
{
	unsigned saved = _mm_getcsr();
	if (j->ftz)
		_mm_setcsr(saved | MXCSR_FTZ_DAZ);
	else
		_mm_setcsr(saved & ~MXCSR_FTZ_DAZ);
	for (int64_t r = j->r0; r < j->r1; ++r) {
		switch (j->kind) {
		case K_RMSNORM:
			rmsnorm_row(j->fo + r * j->n, j->fx + r * j->n, j->fw, j->n, j->eps);
			break;
		case K_ADD_RMSNORM:
			fused_add_rmsnorm_row(j->fo + r * j->n, j->fr + r * j->n, j->fy + r * j->n, j->fw, j->n, j->eps);
			break;
		case K_ROPE: {
			int64_t pos = j->pos0 + r;
			float *tok = j->fr + r * (int64_t)j->heads * j->n;
			const float *cs = j->fc + pos * j->rope_max_dim;
			const float *sn = j->fs + pos * j->rope_max_dim;
			for (int h = 0; h < j->heads; ++h)
				rmsnorm_rope_head(tok + (int64_t)h * j->n, j->n, j->fw, cs, sn, pos, j->eps);
			break;
		}
		case K_ROPE_ONLY: {
			int64_t pos = j->pos0 + r;
			float *tok = j->fr + r * (int64_t)j->heads * j->n;
			const float *cs = j->fc + pos * j->rope_max_dim;
			const float *sn = j->fs + pos * j->rope_max_dim;
			for (int h = 0; h < j->heads; ++h)
				rope_only_head(tok + (int64_t)h * j->n, j->n, cs, sn, pos);
			break;
		}
		case K_ROPE_TABLE: /* rows are positions; n = half, rope_max_dim = row stride */
			rope_table_row(j->fo + r * j->rope_max_dim, j->fr + r * j->rope_max_dim, j->pos0 + r, j->n, j->rope_max_dim, j->freqs);
			break;
		case K_Q8_GEMV:
		case K_Q8_FUSED_GEMV:
		case K_SWIGLU_Q8_GEMV:
		case K_SWIGLU_F32Q8_GEMV: /* rows are (batch, output row) pairs */
			gemv_row(j, r);
			break;
		case K_SWIGLU: /* rows here are chunks of 4096 elements */
		{
			int64_t b = r * 4096, e = b + 4096 < j->n64 ? b + 4096 : j->n64;
			for (int64_t i = b; i < e; ++i)
				j->fo[i] = swiglu_v7(j->fx[i], j->fy[i]);
			break;
		}
		case K_QUANT: {
			int64_t ng = (j->n + ORC_Q8_GS - 1) / ORC_Q8_GS;
			quantize_vec(j->q + r * j->n, j->sc + r * ng, j->fx + r * j->n, j->n);
			break;
		}
		case K_SWIGLU_Q8: {
			float h[ORC_Q8_GS];
			int64_t ng = j->n / ORC_Q8_GS;
			for (int64_t g = 0; g < ng; ++g) {
				int64_t off = r * j->n + g * ORC_Q8_GS;
				for (int i = 0; i < ORC_Q8_GS; ++i)
					h[i] = swiglu_v7(j->fx[off + i], j->fy[off + i]);
				quantize_group64(j->q + off, j->sc + r * ng + g, h);
			}
			break;
		}
		case K_ADD: {
			int64_t b = r * 4096, e = b + 4096 < j->n64 ? b + 4096 : j->n64;
			for (int64_t i = b; i < e; ++i)
				j->fo[i] = j->fo[i] + j->fy[i];
			break;
		}
		case K_RMSNORM_Q8: {
			int64_t ng = j->n / ORC_Q8_GS;
			rmsnorm_quantize_row(j->q + r * j->n, j->sc + r * ng, j->fx + r * j->n, j->fw, j->n, j->eps);
			break;
		}
		case K_SWIGLU_Q8_AVX2:
			swiglu_q8_row_avx2(j->q + r * j->n, j->sc + r * (j->n / ORC_Q8_GS), j->fx + r * j->n, j->fy + r * j->n, j->n);
			break;
		case K_FILL_NORMAL: /* rows relative to dst; pos0 = global index of row 0 */
			fill_normal_row(j->fo + r * j->n64, j->pos0 + r, j->n64, j->seed, j->mean, j->std);
			break;
		}
	}
	_mm_setcsr(saved);
}

static void *thread_main(void *p)
{
	run_job((job *)p);
	return NULL;
}

static int run_rows(const job *proto, int64_t rows, int nthreads)
{
	if (rows <= 0)
		return 0;
	if (nthreads < 1)
		nthreads = 1;
	if (nthreads > 256)
		nthreads = 256;
	if (nthreads > rows)
		nthreads = (int)rows;
	if (nthreads == 1) {
		job j = *proto;
		j.r0 = 0;
		j.r1 = rows;
		run_job(&j);
		return 0;
	}
	job jobs[256];
	pthread_t tid[256];
	for (int t = 0; t < nthreads; ++t) {
		jobs[t] = *proto;
		jobs[t].r0 = rows * t / nthreads;
		jobs[t].r1 = rows * (t + 1) / nthreads;
	}
	for (int t = 1; t < nthreads; ++t) {
		if (pthread_create(&tid[t], NULL, thread_main, &jobs[t]) != 0) {
			/* run the chunk on this thread when no thread can be created */
			run_job(&jobs[t]);
			tid[t] = 0;
		}
	}
	run_job(&jobs[0]);
	for (int t = 1; t < nthreads; ++t)
		if (tid[t])
			pthread_join(tid[t], NULL);
	return 0;
}

/* ------------------------------------------------------------------------ */
/* public entry points                                                       */
/* ------------------------------------------------------------------------ */

int orc_rmsnorm_rows(float *o, const float *x, const float *w, int64_t rows, int n, float eps, int nthreads)
{
	if (n <= 0 || n % 32 != 0 || rows < 0)
		return -1;
	job j = { 0 };
	j.kind = K_RMSNORM;
	j.ftz = 0;
	j.fo = o;
	j.fx = x;
	j.fw = w;
	j.n = n;
	j.eps = eps;
	return run_rows(&j, rows, nthreads);
}

int orc_fused_add_rmsnorm_rows(float *o, float *residual, const float *add, const float *w, int64_t rows, int n, float eps, int nthreads)
{
	if (n <= 0 || n % 8 != 0 || rows < 0)
		return -1;
	job j = { 0 };
	j.kind = K_ADD_RMSNORM;
	j.ftz = 0;
	j.fo = o;
	j.fr = residual;
	j.fy = add;
	j.fw = w;
	j.n = n;
	j.eps = eps;
	return run_rows(&j, rows, nthreads);
}

int orc_rmsnorm_rope_rows(float *buf, int64_t tokens, int n_heads, int head_dim, const float *w, const float *cos_table, const float *sin_table, int64_t pos0, int rope_max_dim, float eps, int nthreads)
{
	if (head_dim <= 0 || head_dim % 32 != 0 || n_heads < 0 || tokens < 0 || pos0 < 0 || rope_max_dim < head_dim / 2)
		return -1;
	job j = { 0 };
	j.kind = K_ROPE;
	j.ftz = 1;
	j.fr = buf;
	j.fw = w;
	j.fc = cos_table;
	j.fs = sin_table;
	j.n = head_dim;
	j.heads = n_heads;
	j.pos0 = pos0;
	j.rope_max_dim = rope_max_dim;
	j.eps = eps;
	return run_rows(&j, tokens, nthreads);
}

float orc_sigmoid(float g)
{
	unsigned saved = _mm_getcsr();
	_mm_setcsr(saved | MXCSR_FTZ_DAZ);
	float r = sigmoid_v7(g);
	_mm_setcsr(saved);
	return r;
}

int orc_swiglu(float *out, const float *g, const float *u, int64_t n, int nthreads)
{
	if (n < 0)
		return -1;
	job j = { 0 };
	j.kind = K_SWIGLU;
	j.ftz = 1;
	j.fo = out;
	j.fx = g;
	j.fy = u;
	j.n64 = n;
	return run_rows(&j, (n + 4095) / 4096, nthreads);
}

int orc_quantize_rows(int8_t *q, float *s, const float *x, int64_t rows, int n, int nthreads)
{
	if (n <= 0 || rows < 0)
		return -1;
	job j = { 0 };
	j.kind = K_QUANT;
	j.ftz = 1;
	j.q = q;
	j.sc = s;
	j.fx = x;
	j.n = n;
	return run_rows(&j, rows, nthreads);
}

int orc_swiglu_q8_rows(int8_t *q, float *s, const float *g, const float *u, int64_t rows, int n, int nthreads)
{
	if (n <= 0 || n % ORC_Q8_GS != 0 || rows < 0)
		return -1;
	job j = { 0 };
	j.kind = K_SWIGLU_Q8;
	j.ftz = 1;
	j.q = q;
	j.sc = s;
	j.fx = g;
	j.fy = u;
	j.n = n;
	return run_rows(&j, rows, nthreads);
}

int orc_add_inplace(float *x, const float *y, int64_t n, int nthreads)
{
	if (n < 0)
		return -1;
	job j = { 0 };
	j.kind = K_ADD;
	j.ftz = 0;
	j.fo = x;
	j.fy = y;
	j.n64 = n;
	return run_rows(&j, (n + 4095) / 4096, nthreads);
}

int orc_rmsnorm_quantize_rows(int8_t *q, float *s, const float *x, const float *w, int64_t rows, int n, float eps, int nthreads)
{
	if (n <= 0 || n % ORC_Q8_GS != 0 || rows < 0)
		return -1;
	job j = { 0 };
	j.kind = K_RMSNORM_Q8;
	j.ftz = 1;
	j.q = q;
	j.sc = s;
	j.fx = x;
	j.fw = w;
	j.n = n;
	j.eps = eps;
	return run_rows(&j, rows, nthreads);
}

int orc_rope_tables(float *cos_table, float *sin_table, int64_t pos0, int64_t positions, int half, int stride, const double *freqs, int nthreads)
{
	if (half <= 0 || stride < half || positions < 0 || pos0 < 0 || pos0 + positions > ((int64_t)1 << 31) || !freqs)
		return -1;
	job j = { 0 };
	j.kind = K_ROPE_TABLE;
	j.ftz = 0;
	j.fo = cos_table;
	j.fr = sin_table;
	j.pos0 = pos0;
	j.n = half;
	j.rope_max_dim = stride;
	j.freqs = freqs;
	return run_rows(&j, positions, nthreads);
}

int orc_rope_only_rows(float *buf, int64_t tokens, int n_heads, int head_dim, const float *cos_table, const float *sin_table, int64_t pos0, int rope_max_dim, int nthreads)
{
	if (head_dim <= 0 || head_dim % 32 != 0 || n_heads < 0 || tokens < 0 || pos0 < 0 || rope_max_dim < head_dim / 2)
		return -1;
	job j = { 0 };
	j.kind = K_ROPE_ONLY;
	j.ftz = 1;
	j.fr = buf;
	j.fc = cos_table;
	j.fs = sin_table;
	j.n = head_dim;
	j.heads = n_heads;
	j.pos0 = pos0;
	j.rope_max_dim = rope_max_dim;
	return run_rows(&j, tokens, nthreads);
}

static int gemv_args_ok(int64_t batch, int n, int d)
{
	return batch >= 0 && d >= 0 && n > 0 && n % ORC_Q8_GS == 0 && n <= ORC_GEMV_MAX_N;
}

int orc_q8_gemv(float *out, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws, int64_t batch, int n, int d, int nthreads)
{
	if (!gemv_args_ok(batch, n, d))
		return -1;
	job j = { 0 };
	j.kind = K_Q8_GEMV;
	j.ftz = 1;
	j.fo = out;
	j.qin = xq;
	j.sin_ = xs;
	j.qw1 = wq;
	j.sw1 = ws;
	j.n = n;
	j.d = d;
	return run_rows(&j, batch * d, nthreads);
}

int orc_q8_fused_gemv(float *out, const float *x, const int8_t *wq, const float *ws, int64_t batch, int n, int d, int nthreads)
{
	if (!gemv_args_ok(batch, n, d))
		return -1;
	job j = { 0 };
	j.kind = K_Q8_FUSED_GEMV;
	j.ftz = 1;
	j.fo = out;
	j.fx = x;
	j.qw1 = wq;
	j.sw1 = ws;
	j.n = n;
	j.d = d;
	return run_rows(&j, batch * d, nthreads);
}

int orc_swiglu_q8_gemv(float *out, const int8_t *xq, const float *xs, const int8_t *gq, const float *gs, const int8_t *uq, const float *us, int64_t batch, int n, int d, int nthreads)
{
	if (!gemv_args_ok(batch, n, d))
		return -1;
	job j = { 0 };
	j.kind = K_SWIGLU_Q8_GEMV;
	j.ftz = 1;
	j.fo = out;
	j.qin = xq;
	j.sin_ = xs;
	j.qw1 = gq;
	j.sw1 = gs;
	j.qw2 = uq;
	j.sw2 = us;
	j.n = n;
	j.d = d;
	return run_rows(&j, batch * d, nthreads);
}

int orc_swiglu_f32q8_gemv(float *out, const float *x, const int8_t *gq, const float *gs, const int8_t *uq, const float *us, int64_t batch, int n, int d, int single_row_path, int nthreads)
{
	if (!gemv_args_ok(batch, n, d))
		return -1;
	job j = { 0 };
	j.kind = K_SWIGLU_F32Q8_GEMV;
	j.ftz = 1;
	j.fo = out;
	j.fx = x;
	j.qw1 = gq;
	j.sw1 = gs;
	j.qw2 = uq;
	j.sw2 = us;
	j.n = n;
	j.d = d;
	j.variant = single_row_path != 0;
	return run_rows(&j, batch * d, nthreads);
}

int orc_fill_normal(float *dst, int64_t rows, int64_t n, int64_t row0, uint64_t seed, float mean, float std, int nthreads)
{
	if (rows < 0 || n < 0 || row0 < 0 || (!dst && rows && n))
		return -1;
	if (rows == 0 || n == 0)
		return 0;
	job j = { 0 };
	j.kind = K_FILL_NORMAL;
	j.ftz = 0;
	j.fo = dst;
	j.n64 = n;
	j.pos0 = row0;
	j.seed = seed;
	j.mean = mean;
	j.std = std;
	return run_rows(&j, rows, nthreads);
}

int orc_swiglu_q8_rows_avx2(int8_t *q, float *s, const float *g, const float *u, int64_t rows, int n, int nthreads)
{
	if (n <= 0 || n % ORC_Q8_GS != 0 || rows < 0)
		return -1;
	job j = { 0 };
	j.kind = K_SWIGLU_Q8_AVX2;
	j.ftz = 1;
	j.q = q;
	j.sc = s;
	j.fx = g;
	j.fy = u;
	j.n = n;
	return run_rows(&j, rows, nthreads);
}
