/* v7g.h -- row-batched, device-resident C-ABI of the B200 (sm_100a) kernels.
 *
 * These entry points are the batched form of v7's per-vector kernels: where the
 * reference normalises ONE row (or one token's heads) per call on the CPU, each
 * entry here processes `rows` independent rows of device memory in one kernel
 * launch on `stream` (a cudaStream_t passed as void*, NULL = legacy default
 * stream).  All pointers are device pointers on the current CUDA device; the
 * caller owns every buffer and nothing is allocated.  Calls are asynchronous:
 * results are ready once `stream` has been synchronised.
 *
 * Layout (row-major, contiguous rows):
 *   activations  float [rows, n]
 *   gamma        float [n]           (shared by all rows / all heads)
 *   Q8 codes     int8  [rows, n]     (v7_q8_tensor.q, src/v7_lib.h:52-56)
 *   Q8 scales    float [rows, ceil(n/64)]  one absmax scale per 64-element
 *                                    group, row order (src/q8_batch4.h:15-19)
 *
 * Return value: V7G_OK (0) or a V7G_ERR_* code; v7g_last_error() gives the
 * message of the calling thread's last failure.  A contract violation is
 * reported before anything is launched and leaves every output untouched.
 *
 * The arithmetic of every kernel reproduces the reference's AVX2 kernel
 * operation for operation (same rounding steps, same reduction order), so the
 * results match v7's own library bit for bit on the same input bytes.
 */
#ifndef V7G_H
#define V7G_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum v7g_status {
	V7G_OK = 0,
	V7G_ERR_ARG = 1,         /* argument breaks the kernel contract */
	V7G_ERR_CUDA = 2,        /* a CUDA runtime call failed */
	V7G_ERR_UNSUPPORTED = 3, /* shape outside what this build implements */
	V7G_ERR_NO_DEVICE = 4    /* no usable sm_100 device */
};

/* A1  RMSNorm rows: o[r] = (x[r] * s_r) * w with s_r = 1/sqrt(sum(x[r]^2)/n + eps).
   Replaces a loop of v7s_rmsnorm (src/v7_lib.h:270, rmsnorm_kernel.inc:12-75).
   Contract: n > 0, n % 32 == 0.  o may alias x. */
int v7g_rmsnorm_rows(float *o, const float *x, const float *w, int64_t rows, int n, float eps, void *stream);

/* A2  fused residual-add + RMSNorm rows: residual[r] += add[r] (written back),
   o[r] = rmsnorm(residual[r]) * w.  Replaces a loop of v7s_fused_add_rmsnorm
   (src/v7_lib.h:272, add_rmsnorm_kernel.inc:15-129).  Contract: n > 0, n % 8 == 0. */
int v7g_fused_add_rmsnorm_rows(float *o, float *residual, const float *add, const float *w, int64_t rows, int n, float eps, void *stream);

/* A3  per-head RMSNorm + NeoX half-split RoPE over GQA Q/K, in place.
   q [tokens, n_q_heads, head_dim], k [tokens, n_kv_heads, head_dim]; token t is
   at position pos0 + t and reads cos/sin row (pos0 + t) * rope_max_dim (first
   head_dim/2 entries).  Position 0 normalises without rotating.  Replaces, per
   token, v7s_rmsnorm_rope_heads on Q then on K (src/v7_lib.h:273,
   rmsnorm_rope_dispatch.inc:11-52, forward_q8.inc:339-343).
   Contract: head_dim % 32 == 0, 32 <= head_dim <= 1024, rope_max_dim >= head_dim/2.
   Either tensor may be NULL with a head count of 0. */
int v7g_rmsnorm_rope_rows(float *q, float *k, int64_t tokens, int n_q_heads, int n_kv_heads, int head_dim, const float *wq, const float *wk, const float *cos_table, const float *sin_table, int64_t pos0, int rope_max_dim, float eps, void *stream);

/* A5  elementwise SwiGLU: out = (sigmoid(gate) * gate) * up over `count`
   elements, with v7's polynomial sigmoid (EVAL_SIGMOID, v7_macros.inc:98-160)
   and its product order (swiglu_q8_kernel.inc:204-209).  out may alias gate or up. */
int v7g_swiglu(float *out, const float *gate, const float *up, int64_t count, void *stream);

/* A8  SwiGLU then Q8 requantisation per row, the SwiGLU value never leaving
   registers: codes [rows, n], scales [rows, n/64].  The quantiser follows
   v7d_quantize (utility_dispatch.inc:110-213, quantize_kernel.inc:43-159).
   Contract: n > 0, n % 64 == 0. */
int v7g_swiglu_q8_rows(int8_t *codes, float *scales, const float *gate, const float *up, int64_t rows, int n, void *stream);

/* A6  Q8 quantisation of `rows` vectors of n floats: codes [rows, n], scales
   [rows, ceil(n/64)].  A trailing group shorter than 64 takes the reference's
   scalar tail rule.  Replaces a loop of v7d_quantize (src/v7_lib.h:123). */
int v7g_quantize_rows(int8_t *codes, float *scales, const float *x, int64_t rows, int n, void *stream);

/* A7  x += y over `count` floats.  Replaces v7s_add_inplace (src/v7_lib.h:271,
   add_kernel.inc:26-49). */
int v7g_add_inplace(float *x, const float *y, int64_t count, void *stream);

/* Fused RMSNorm -> Q8 per row (v7s_rmsnorm_quantize, src/v7_lib.h:124,
   rmsnorm_quantize_kernel.inc:60-218): codes [rows, n], scales [rows, n/64].
   Contract: n > 0, n % 64 == 0. */
int v7g_rmsnorm_quantize_rows(int8_t *codes, float *scales, const float *x, const float *w, int64_t rows, int n, float eps, void *stream);

/* RoPE without the norm over GQA Q/K, in place (v7s_rope_only_heads,
   rope_only_kernel.inc:11-53, rope_only_dispatch.inc:10-47; the path of
   models without a QK norm, forward_q8.inc:40-44).  Same layout and table
   addressing as v7g_rmsnorm_rope_rows; position 0 leaves its heads untouched.
   Contract: head_dim % 32 == 0, 32 <= head_dim <= 1024. */
int v7g_rope_only_rows(float *q, float *k, int64_t tokens, int n_q_heads, int n_kv_heads, int head_dim, const float *cos_table, const float *sin_table, int64_t pos0, int rope_max_dim, void *stream);

/* RoPE frequencies freqs[j], j < half (host function, host memory, no
   device): base^(-j/half) as the reference's table builder computes it on
   the x87 unit and stores it as a double (fused_f32_kernel.inc:117-147), or
   with llama3 scaling when scaling == 1 (:149-256; factor, high/low frequency
   factors and original context length as in the keys __sys_rope_factor,
   __sys_rope_high_freq_factor, __sys_rope_low_freq_factor,
   __sys_rope_orig_max_pos).  Contract: 0 < half <= 256. */
int v7g_rope_freqs(double *freqs, int half, float base, int scaling, float factor, float high_freq_factor, float low_freq_factor, int orig_max_pos);

/* RoPE tables on the device: rows pos0 .. pos0+positions-1 of cos / sin,
   row stride `stride` floats, entry j < half = cos / sin(freqs[j] * pos) with
   the angle at x87 extended precision (fused_f32_kernel.inc:257-302),
   columns half.. zero.  freqs: HOST array of `half` doubles (v7g_rope_freqs).
   Agrees with the reference's fsincos tables to within one fp32 ulp (equal
   on all but about one entry in ten million).
   Contract: 0 < half <= 256, stride >= half, pos0 + positions <= 2^31. */
int v7g_rope_tables(float *cos_table, float *sin_table, int64_t pos0, int64_t positions, int half, int stride, const double *freqs, void *stream);

/* Positions of the tables v7s_rope_init builds (ROPE_INTERNAL_MAX_SEQ_LEN,
   fused_f32_kernel.inc:9). */
#define V7G_ROPE_TABLE_POSITIONS 131072

/* Builds the library's RoPE tables [V7G_ROPE_TABLE_POSITIONS, head_dim/2] on
   the current device from explicit parameters (v7s_rope_init reads the same
   ones from the key store): v7g_rope_freqs on the host, then v7g_rope_tables.
   Synchronous.  Contract: head_dim even, head_dim/2 <= 256. */
int v7g_rope_init(int head_dim, float base, int scaling, float factor, float high_freq_factor, float low_freq_factor, int orig_max_pos);

/* The device tables the last v7s_rope_init / v7g_rope_init built on the current device:
   [V7G_ROPE_TABLE_POSITIONS, *half] fp32 each, row stride *half, owned by the
   library (freed by v7s_shutdown).  V7G_ERR_ARG when none was built. */
int v7g_get_rope_tables(const float **cos_table, const float **sin_table, int *half);

/* ---- Q8-weight matrix-vector products ----------------------------------
   Weights: codes [d, n] int8 row-major (4-byte aligned) + scales [d, n/64]
   fp32, one per 64-element group of a row (src/q8_batch4.h:15-19).  batch
   activation vectors of n; out [batch, d] fp32.  Contract: n > 0,
   n % 64 == 0, n <= 65536, batch <= 65535.  Weight bytes in [-127, 127] (the
   exporter's contract); a -128 weight is multiplied as the reference's
   vpsignb forms it.  Every output equals the reference's bit for bit.
   v7g_q8_gemv and v7g_swiglu_q8_gemv with batch >= 2 stream the weights once
   per block of 2 or 4 activation rows, as the reference's four-token
   v7d_q8_batch4 does (src/q8_batch4.h:5-19, q8_batch4_kernel.inc:5-10); each
   row's result is its one-row result. */

/* v7d_q8 (src/v7_lib.h:113, q8_kernel.inc:84-207): out[b, i] = dot(x_b, w_i),
   x Q8: codes [batch, n] (16-byte aligned) + scales [batch, n/64]. */
int v7g_q8_gemv(float *out, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws, int64_t batch, int n, int d, void *stream);

/* v7d_q8_fused (fused_dispatch.inc:82-114): each fp32 activation x [batch, n]
   quantised with v7d_quantize's rules, then v7d_q8 -- in one kernel. */
int v7g_q8_fused_gemv(float *out, const float *x, const int8_t *wq, const float *ws, int64_t batch, int n, int d, void *stream);

/* v7d_swiglu_q8 (src/v7_lib.h:117, swiglu_q8_kernel.inc:16-286):
   out[b, i] = swiglu(dot(x_b, gate_i), dot(x_b, up_i)), Q8 activation. */
int v7g_swiglu_q8_gemv(float *out, const int8_t *xq, const float *xs, const int8_t *gate_q, const float *gate_s, const int8_t *up_q, const float *up_s, int64_t batch, int n, int d, void *stream);

/* v7d_swiglu (src/v7_lib.h:116, swiglu_kernel.inc): fp32 activation x
   [batch, n] times Q8 gate/up, SwiGLU epilogue, with the arithmetic of the
   reference's dual-row path (every row of an even-sized work chunk; the
   reference's single-row path for the last row of an odd-sized chunk groups
   the sums differently and can differ in the last bits). */
int v7g_swiglu_f32q8_gemv(float *out, const float *x, const int8_t *gate_q, const float *gate_s, const int8_t *up_q, const float *up_s, int64_t batch, int n, int d, void *stream);

/* Number of bounded waits in the pipelined GEMV kernels that gave up since
   the library was loaded (a kernel that gives up writes no result for the
   rows it was computing).  0 in every correct run; 0xffffffff when the
   counter cannot be read. */
unsigned int v7g_pipeline_timeouts(void);

/* RMSNorm rows on HOST buffers with no device allocation.  No counterpart in
   the reference: it is the host-buffer path of v7s_rmsnorm for callers that
   must not have a library allocate device memory -- a program that shares the
   GPU with a framework whose caching allocator holds nearly all of it, a
   latency-critical loop that cannot take the device-wide synchronisation of
   cudaMalloc / cudaFree, or a deployment that forbids allocation after
   start-up.  o, x [rows, n] and w [n] may be host (pageable or pinned) or
   device memory; they are staged through a static device array of
   V7G_NOALLOC_SCRATCH_BYTES that every GPU loading the library holds until the
   process exits.  Work beyond that (gamma plus x and o, each rounded up to 256
   bytes) is rejected with V7G_ERR_ARG.  The first call on a device looks up
   the array's device address (cudaGetSymbolAddress) and keeps it until the
   process exits, so make that call before any stream capture, and do not
   call cudaDeviceReset in between.  `stream` must belong to the current
   device (V7G_ERR_ARG otherwise).  Synchronous: returns when o is written,
   and on a failure only once nothing it queued is still running.  Calls
   share the array; they are serialised and each waits for `stream`, so they
   never overlap on the GPU -- calls that did overlap would race.  Nothing
   needs clearing between calls: each copies its whole input in and output
   out.  Results equal v7g_rmsnorm_rows bit for bit.  Contract: n % 32 == 0. */
#define V7G_NOALLOC_SCRATCH_BYTES (4u << 20)
int v7g_rmsnorm_rows_noalloc(float *o, const float *x, const float *w, int64_t rows, int n, float eps, void *stream);

/* ---- runtime ---------------------------------------------------------- */

/* RMS epsilon used by the reference-ABI entries (v7s_rmsnorm & co.), which
   take no eps argument.  The reference reads it from the BSS global g_rms_eps,
   set from the DB key __sys_rms_eps (inf_microdb.inc:49-53); it is 0 until set. */
void v7g_set_rms_eps(float eps);
float v7g_get_rms_eps(void);

/* Message of the calling thread's last failed call ("" when none). */
const char *v7g_last_error(void);

/* Number of kernels this library has launched in this process. */
uint64_t v7g_launch_count(void);

/* Launch overlap (programmatic dependent launch), on by default: each kernel
   is launched so that it may be scheduled while the kernel ahead of it in the
   stream drains, and waits on the device for that kernel's completion before
   its first memory access.  Stream order is kept either way; off gives plain
   launches.  Process-wide; takes effect at the next launch.  The environment
   variable V7G_LAUNCH_OVERLAP=0, read when the library is loaded, starts it
   off.  No reference counterpart (the reference's kernels are CPU calls). */
void v7g_set_launch_overlap(int on);
int v7g_get_launch_overlap(void);

/* Exhaustive device self-check of the library's fast arithmetic (the
   Markstein-corrected reciprocal, the fast Q8 scale, the packed-pair SiLU and
   Q8 code paths) against the plain IEEE instructions, over every input each can
   receive, plus 2^31 Q8 products next to a rounding tie (where fusing the
   product into the rounding step would show).  dev_counts: 7 zeroed device
   counters, incremented by the number of mismatches of each test (all must
   stay 0).  Asynchronous on `stream`. */
int v7g_selftest_arith(unsigned long long *dev_counts, void *stream);

/* Library version string. */
const char *v7g_version(void);

/* Deterministic synthetic input: dst[r, j] ~ N(mean, std) for r in [0, rows),
   j in [0, n), generated from (seed, row0 + r, j) alone, so any row shard of a
   larger matrix is reproducible independently on any device.  Box-Muller over
   a SplitMix64 counter hash, evaluated with correctly rounded IEEE operations
   only (no math-library calls), so a host program doing the same operations
   reproduces every value bit for bit. */
int v7g_fill_normal(float *dst, int64_t rows, int64_t n, int64_t row0, uint64_t seed, float mean, float std, void *stream);

#ifdef __cplusplus
}
#endif
#endif
