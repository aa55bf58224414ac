/* v7_threading.h -- the drop-in export surface of libv7_threading.so.
 *
 * The reference's host loader (src/v7_lib.h:585-739, v7_load) dlopens
 * libv7_threading.so and resolves 99 names with dlsym, exiting on the first one
 * missing.  Every function is called with the Microsoft x64 convention
 * (src/v7_lib.h:40-46: __attribute__((ms_abi)) on Linux).  This library exports
 * the same 99 names with the same convention, so the reference's loadtests and
 * validators (tools/b_*_loadtest.cpp, tools/v_*_validate.cpp) run unchanged
 * against it.
 *
 * The v7 hot path (the elementwise / reduction kernels) is implemented on the
 * GPU: each entry accepts HOST or DEVICE pointers (decided per pointer with
 * cudaPointerGetAttributes).  Device pointers are used in place; host buffers
 * are staged through a device workspace.  Every call returns with its results
 * written, as the reference's do.  The calls take no stream, so a call given
 * any device pointer first waits for all work already queued on that device
 * (cudaDeviceSynchronize): inputs a caller's kernel is still writing, on any
 * stream, are complete before they are read.  A call leaves the calling
 * thread's current CUDA device as it found it.
 *
 * Everything outside that path (models, chat, tokenizer, attention, matmul,
 * vision, SectorLogo, ...) is exported as a stub: it returns 0/NULL and marks
 * the engine dead with a reason, which v7_engine_is_dead() /
 * v7_get_death_reason() report (the reference's FATAL contract,
 * src/v7_lib.h:179-184).  See v7_threading_stubs.h for that list.
 */
#ifndef V7_THREADING_H
#define V7_THREADING_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__linux__) && defined(__x86_64__)
#define V7_ABI __attribute__((ms_abi))
#else
#define V7_ABI
#endif

/* Data layouts shared with the reference (src/v7_lib.h:52-62). */
typedef struct v7_q8_tensor {
	char *q;  /* int8 codes */
	float *s; /* one fp32 scale per 64-element group */
} v7_q8_tensor;
typedef struct v7_f32_tensor {
	float *data;
	float *scales;
} v7_f32_tensor;
/* Opaque here: only passed through by the stubs. */
struct v7_run_state;
struct v7_config;
struct inference_context;
struct v7_probindex;

/* ---- hot path, implemented on the GPU --------------------------------- */

/* src/v7_lib.h:270; rmsnorm_kernel.inc:12-75.  o = (x*scale)*w for one row;
   size % 32 == 0.  eps = the library's RMS epsilon (v7g_set_rms_eps /
   ht_add("__sys_rms_eps")). */
V7_ABI void v7s_rmsnorm(float *o, float *x, float *weight, int size);
/* src/v7_lib.h:271; add_kernel.inc:26-49.  x += y; n % 32 == 0. */
V7_ABI void v7s_add_inplace(float *x, float *y, int n);
/* src/v7_lib.h:272; add_rmsnorm_kernel.inc:15-129.  residual += add (in place),
   o = rmsnorm(residual)*weight; dim % 8 == 0. */
V7_ABI void v7s_fused_add_rmsnorm(float *o, float *residual, float *add, float *weight, int dim);
/* src/v7_lib.h:273; rmsnorm_rope_dispatch.inc:11-52.  One token's n_heads
   heads, in place, position pos; head_dim % 32 == 0. */
V7_ABI void v7s_rmsnorm_rope_heads(float *buf, int n_heads, int head_dim, float *norm_weight, float *cos_table, float *sin_table, int pos, int rope_max_dim);
/* src/v7_lib.h:123; utility_dispatch.inc:110-213.  Q8 quantisation of n floats. */
V7_ABI void v7d_quantize(char *out_q, float *in_x, float *out_s, int n);
/* src/v7_lib.h:124; rmsnorm_quantize_kernel.inc:60-218.  RMSNorm then Q8;
   n % 64 == 0. */
V7_ABI void v7s_rmsnorm_quantize(char *out_q, float *in_x, float *out_s, int n, float *weight);

/* src/v7_lib.h:113; q8_kernel.inc:84-207, matmul_dispatch.inc.  xout[i] =
   dot(x, row i of w) for i < d: Q8 activation (x->q [n], x->s [n/64]) times Q8
   weights (w->q [d, n], w->s [d, n/64]); n % 64 == 0. */
V7_ABI void v7d_q8(float *xout, v7_q8_tensor *x, v7_q8_tensor *w, int n, int d);
/* src/v7_lib.h:116; swiglu_kernel.inc, fused_dispatch.inc:27-57.  xout[i] =
   swiglu(dot(x, gate row i), dot(x, up row i)), fp32 activation x->data [n];
   n % 64 == 0.  Arithmetic of the reference's dual-row path. */
V7_ABI void v7d_swiglu(float *xout, v7_f32_tensor *x, v7_q8_tensor *gate_w, int n, int d, v7_q8_tensor *up_w);
/* src/v7_lib.h:117; swiglu_q8_kernel.inc:16-286.  As v7d_swiglu with a Q8
   activation; n % 64 == 0. */
V7_ABI void v7d_swiglu_q8(float *xout, v7_q8_tensor *x, v7_q8_tensor *gate_w, int n, int d, v7_q8_tensor *up_w);

/* ---- engine-internal kernels ------------------------------------------- */
/* The reference links these statically into its forward pass; they are not
   among the names v7_load resolves.  Exported here under the same names and
   conventions so that an engine-side caller can bind them. */

/* Argument block of the four-token Q8 GEMV (src/q8_batch4.h:29-38), 120
   bytes: four output arrays [d], four Q8 activations (codes [n], scales
   [n/64]), one Q8 weight matrix (codes [d, n], scales [d, n/64]). */
typedef struct v7_q8_batch4_args {
	float *out[4];        /* byte offset 0 */
	const int8_t *xq[4];  /* 32 */
	const float *xs[4];   /* 64 */
	const int8_t *wq;     /* 96 */
	const float *ws;      /* 104 */
	uint32_t n;           /* 112: n % 64 == 0 */
	uint32_t d;           /* 116 */
} v7_q8_batch4_args;

/* v7_threading.def:13-14, src/q8_batch4.h:40-41; q8_batch4_kernel.inc:5-10
   (called from prefill_q8.inc:630).  Four v7d_q8 products of one weight
   matrix: out[t][i] = dot(token t, row i of w), each token's result equal to
   its own v7d_q8 result; the weights are streamed once for the four tokens.
   v7s_ is the reference's single-thread kernel, v7d_ its dispatched form;
   here both run the same GPU kernel.  Host or device pointers, as v7d_q8. */
V7_ABI void v7s_q8_batch4(const v7_q8_batch4_args *args);
V7_ABI void v7d_q8_batch4(const v7_q8_batch4_args *args);

/* rope_only_dispatch.inc:10-47 (called at forward_q8.inc:44).  RoPE without
   the norm on one token's n_heads heads, in place; cos/sin row
   pos * rope_max_dim; position 0 is the identity; head_dim % 32 == 0. */
V7_ABI void v7s_rope_only_heads(float *buf, int n_heads, int head_dim, float *cos_table, float *sin_table, int pos, int rope_max_dim);

/* Descriptor of v7s_qk_fork_heads (qk_fork_kernel.inc:10-27), 48 bytes. */
typedef struct v7_qk_fork_args {
	float *buf;    /* first head */
	float *weight; /* per-layer norm gamma [head_dim] */
	float *cos;    /* cos table, already offset to the position's row */
	float *sin;    /* sin table, already offset to the position's row */
	int head_dim;
	int heads;
	int pos;
	int unused;
} v7_qk_fork_args;

/* qk_fork_kernel.inc:40-62: the RMSNorm + RoPE of v7s_rmsnorm_rope_heads over
   args->heads heads, every input taken from the descriptor (reentrant in the
   reference). */
V7_ABI void v7s_qk_fork_heads(const v7_qk_fork_args *args);

/* ---- runtime surface, implemented on the host ------------------------- */

V7_ABI int v7_init(const char *db_path);                 /* src/v7_lib.h:167 */
V7_ABI int v7_db_load(const char *path);                 /* :168 */
V7_ABI int v7_db_save(const char *path);                 /* :169 */
V7_ABI int v7_engine_is_dead(void);                      /* :183 */
V7_ABI const char *v7_get_death_reason(void);            /* :184 */
V7_ABI const char *v7_get_version(void);                 /* :185 */
V7_ABI int v7_get_console_width(void);                   /* :189 */
V7_ABI int v7_db_add(const char *key, const void *data, int len, unsigned int persist); /* :238 */
V7_ABI void *v7_db_find(const char *key, unsigned long long *out_len);                 /* :239 */
V7_ABI void v7_shutdown(void);                           /* :250 */
/* :275; fused_dispatch.inc:58-76.  Builds the library's RoPE tables
   [131072, head_dim/2] on the current device (v7g_get_rope_tables) from the
   keys __sys_rope_base (float) and __sys_rope_type (int; 1 = llama3, which
   also reads __sys_rope_factor, __sys_rope_high_freq_factor,
   __sys_rope_low_freq_factor, __sys_rope_orig_max_pos).  A missing key marks
   the engine dead, as the reference FATALs.  rope_base is not read (the
   reference takes the base from the key store too). */
V7_ABI void v7s_rope_init(int head_dim, float rope_base);
V7_ABI void v7s_set_fused_rope(int pos, int head_dim);   /* :276; records the position */
V7_ABI void v7s_set_spin(int flag);                      /* :278 */
V7_ABI void v7s_enable_thinking(int on);                 /* :279 */
V7_ABI void v7s_shutdown(void);                          /* :280 */
V7_ABI int v7s_get_num_workers(void);                    /* :281 */
V7_ABI unsigned long long get_config_was_fixed(void);    /* :283 */
V7_ABI void v7_do_fatal(const char *message);            /* :303 */
V7_ABI void ht_init(void);                               /* :130 */
V7_ABI void ht_destroy(void);                            /* :131 */
V7_ABI int ht_add(const char *key, void *data, unsigned long long data_len, unsigned int persist); /* :132 */
V7_ABI void *ht_find(const char *key, unsigned long long *out_len);                               /* :133 */
V7_ABI int db_save(const char *filename);                /* :134 */
V7_ABI int db_load(const char *filename);                /* :135 */
V7_ABI void db_set_readonly(int flag);                   /* :138 */

/* Exported but not provided: marks the engine dead ("v7sprintf: not provided
   by v7g") and returns 0.  Declared here rather than in v7_threading_stubs.h
   because it is variadic. */
V7_ABI int v7sprintf(char *buffer, int buf_size, const char *format, ...); /* :318 */

/* Exported data words (src/v7_lib.h:306-314). */
extern int enable_token_dump;
extern int enable_dump;
extern int cpu_features_ok;

#ifdef __cplusplus
}
#endif

#include "v7_threading_stubs.h"

#endif
