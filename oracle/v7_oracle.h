/* v7_oracle.h -- CPU restatement of v7's elementwise / reduction kernels.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * sm_100a kernels in v7multiplikator_b200/csrc.  Only tests/, the smoke() entry
 * of __graft_entry__.py and the CPU-baseline leg of bench.py may load or call
 * it; no product code path links against it, and the product library fails
 * loudly instead of falling back to it.
 *
 * Every function restates the arithmetic of the reference's NASM/AVX2 kernel
 * (cpki-gmbh/v7multiplikator v2.36.8) operation for operation, so that the
 * result is the one the reference's own library would produce for the same
 * input bytes:
 *   - the 4 x 8 FMA accumulator layout of the sum of squares and the
 *     HADD_YMM addition tree (rmsnorm_kernel.inc:22-46, v7_macros.inc:38-45),
 *   - the exact-IEEE RMS scale 1/sqrt(ss/n + eps) (v7_macros.inc:348-354),
 *   - x86 MAXPS/MINPS operand semantics (the second operand is returned when
 *     either input is NaN), CVTPS2DQ (NaN/overflow -> INT_MIN) followed by the
 *     saturating packs and the -127 floor (quantize_kernel.inc:62-106),
 *   - the MXCSR state each kernel runs under: the dispatched kernels
 *     (RMSNorm+RoPE, quantize, the SwiGLU epilogue) run with FTZ+DAZ
 *     (v7_init.inc:103-109, rmsnorm_rope_dispatch.inc:37,
 *     utility_dispatch.inc:127); the direct-call kernels (RMSNorm, fused
 *     add+RMSNorm, add_inplace) run with the caller's default MXCSR.
 *
 * Row-batched entry points split rows over `nthreads` POSIX threads (rows are
 * independent, so the result does not depend on the thread count).
 * All functions return 0 on success and a negative value when the arguments
 * break the kernel contract the reference states.
 */
#ifndef V7_ORACLE_H
#define V7_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* group size of the Q8 layout (src/q8_batch4.h:15-19) */
#define ORC_Q8_GS 64
/* group-max floor 127 * 2^-126: makes the all-zero-group scale FLT_MIN
   (quantize_kernel.inc:40-41) */
#define ORC_Q8_WMAX_FLOOR 1.4928778e-36f

/* A1  v7s_rmsnorm per row: o = (x * scale) * w, scale = 1/sqrt(ss/n + eps).
   Contract n % 32 == 0 (rmsnorm_kernel.inc:15-20). */
int orc_rmsnorm_rows(float *o, const float *x, const float *w, int64_t rows, int n, float eps, int nthreads);

/* A2  v7s_fused_add_rmsnorm per row: residual += add (stored back in place),
   o = (residual * scale) * w.  Contract n % 8 == 0; leftover blocks
   (n/8 % 4) feed accumulator A first (add_rmsnorm_kernel.inc:37-43,112-121). */
int orc_fused_add_rmsnorm_rows(float *o, float *residual, const float *add, const float *w, int64_t rows, int n, float eps, int nthreads);

/* A3  v7s_rmsnorm_rope_heads over `tokens` tokens of one tensor laid out
   [tokens, n_heads, head_dim], in place.  Token t uses position pos0 + t and
   the cos/sin table row (pos0 + t) * rope_max_dim.  Position 0 normalises
   only (v7_macros.inc:293-295).  Contract head_dim % 32 == 0. FTZ+DAZ. */
int orc_rmsnorm_rope_rows(float *buf, int64_t tokens, int n_heads, int head_dim, const float *w, const float *cos_table, const float *sin_table, int64_t pos0, int rope_max_dim, float eps, int nthreads);

/* A5  EVAL_SIGMOID (v7_macros.inc:98-160) of one value under FTZ+DAZ. */
float orc_sigmoid(float g);

/* A5  elementwise SwiGLU out = (sigmoid(g) * g) * u over n elements.
   FTZ+DAZ, product order of swiglu_q8_kernel.inc:204-209. */
int orc_swiglu(float *out, const float *g, const float *u, int64_t n, int nthreads);

/* A6  v7d_quantize of `rows` independent vectors of n floats each:
   codes [rows, n] int8, scales [rows, ceil(n/64)] fp32.  A trailing group of
   fewer than 64 elements follows the scalar tail path
   (quantize_kernel.inc:119-152).  FTZ+DAZ. */
int orc_quantize_rows(int8_t *q, float *s, const float *x, int64_t rows, int n, int nthreads);

/* A8  SwiGLU followed by Q8 quantisation per row (the SwiGLU result is never
   stored).  Contract n % 64 == 0.  FTZ+DAZ. */
int orc_swiglu_q8_rows(int8_t *q, float *s, const float *g, const float *u, int64_t rows, int n, int nthreads);

/* A7  v7s_add_inplace: x += y over n elements (add_kernel.inc:26-49). */
int orc_add_inplace(float *x, const float *y, int64_t n, int nthreads);

/* Next row 1: v7s_rmsnorm_quantize per row: RMSNorm (A1 arithmetic) then Q8
   quantisation of the normalised row; equal by contract to the
   v7s_rmsnorm -> v7d_quantize chain (tools/kt_utils.h:850-932).
   Contract n % 64 == 0. */
int orc_rmsnorm_quantize_rows(int8_t *q, float *s, const float *x, const float *w, int64_t rows, int n, float eps, int nthreads);

/* Next row 2: RoPE without the norm (v7s_rope_only_heads,
   rope_only_kernel.inc:11-53, rope_only_dispatch.inc:10-47) over `tokens`
   tokens of one tensor [tokens, n_heads, head_dim], in place.  Position 0
   is the identity.  Contract head_dim % 32 == 0.  FTZ+DAZ. */
int orc_rope_only_rows(float *buf, int64_t tokens, int n_heads, int head_dim, const float *cos_table, const float *sin_table, int64_t pos0, int rope_max_dim, int nthreads);

/* largest half the reference's frequency buffer holds (256 doubles,
   fused_f32_kernel.inc:138-139) */
#define ORC_ROPE_MAX_HALF 256

/* A4 frequencies freqs[j], j < half, as the reference's table builder
   computes and stores them (doubles): base^(-j/half) by the x87 chain of
   fused_f32_kernel.inc:120-137 (scaling 0), or with llama3 scaling
   (scaling 1, :149-256; factor, high/low frequency factors and the original
   context length as the __sys_rope_* keys hold them). */
int orc_rope_freqs(double *freqs, int half, float base, int scaling, float factor, float high_freq_factor, float low_freq_factor, int orig_max_pos);

/* A4 tables: rows pos0 .. pos0+positions-1 of cos / sin (row stride `stride`,
   columns half.. zero): angle = freqs[j] * pos at x87 extended precision,
   fsincos, stored as fp32 (fused_f32_kernel.inc:257-302). */
int orc_rope_tables(float *cos_table, float *sin_table, int64_t pos0, int64_t positions, int half, int stride, const double *freqs, int nthreads);

/* ---- Q8-weight GEMVs (next rows 3 and 4) -------------------------------
   Weights: codes [d, n] int8 row-major, scales [d, n/64]; activations: batch
   vectors of n (codes [batch, n] + scales [batch, n/64], or fp32 [batch, n]);
   out [batch, d].  Contract n % 64 == 0 (FATAL-guarded in the reference),
   n <= ORC_GEMV_MAX_N.  FTZ+DAZ (dispatched kernels).  Weight bytes are
   expected in [-127, 127] (the exporter's contract); -128 is multiplied the
   way vpsignb forms it, as the reference does. */
#define ORC_GEMV_MAX_N 65536

/* v7d_q8 (q8_kernel.inc:84-207): out = sum of the 8 lane accumulators. */
int orc_q8_gemv(float *out, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws, int64_t batch, int n, int d, int nthreads);

/* v7d_q8_fused (fused_dispatch.inc:82-114): v7d_quantize of each fp32
   activation vector, then v7d_q8. */
int orc_q8_fused_gemv(float *out, const float *x, const int8_t *wq, const float *ws, int64_t batch, int n, int d, int nthreads);

/* v7d_swiglu_q8 (swiglu_q8_kernel.inc:16-286): gate and up Q8 x Q8 dots,
   then (sigmoid(g) * g) * u with EVAL_SIGMOID. */
int orc_swiglu_q8_gemv(float *out, const int8_t *xq, const float *xs, const int8_t *gq, const float *gs, const int8_t *uq, const float *us, int64_t batch, int n, int d, int nthreads);

/* v7d_swiglu (swiglu_kernel.inc): fp32 activations x Q8 weights, then the
   SwiGLU epilogue.  single_row_path = 0: the dual-row arithmetic (every row of
   an even-sized work chunk); 1: the single-row arithmetic the reference uses
   for the last row of an odd-sized chunk. */
int orc_swiglu_f32q8_gemv(float *out, const float *x, const int8_t *gq, const float *gs, const int8_t *uq, const float *us, int64_t batch, int n, int d, int single_row_path, int nthreads);

/* orc_swiglu_q8_rows in AVX2 (eight lanes per instruction, the reference's
   own instruction forms): identical bits, several times faster; the CPU
   baseline times this form.  n % 64 == 0. */
int orc_swiglu_q8_rows_avx2(int8_t *q, float *s, const float *g, const float *u, int64_t rows, int n, int nthreads);

/* The library's synthetic-input generator v7g_fill_normal restated on the
   CPU (not reference code): dst[r, c] ~ N(mean, std) for global row row0 + r,
   bit-identical to the device's values for the same (seed, row, column). */
int orc_fill_normal(float *dst, int64_t rows, int64_t n, int64_t row0, uint64_t seed, float mean, float std, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
