/* abi_shim.c -- the CPU oracle behind the reference's export surface.
 *
 * TEST INFRASTRUCTURE ONLY.  Builds libv7_oracle_abi.so, which exports the 99
 * names the reference's loader resolves (src/v7_lib.h:585-739) with the ms_abi
 * convention, the hot-path kernels computed by the oracle on host memory.
 * Its one purpose: run the reference's own validators (tools/v_rmsnorm_validate,
 * v_add_inplace_validate, v_quantize_validate, built from the reference's
 * sources into oracle/_ref/) against the oracle, which pins the restatement to
 * the reference's C references, seeds and tolerances.  Never shipped.
 */
#include "v7_threading.h"
#include "v7_oracle.h"

#include <stdio.h>
#include <string.h>

unsigned long long v7g_zero_block[16];
int enable_token_dump;
int enable_dump;
int cpu_features_ok = 1;

/* The kernels' RMS epsilon; "__sys_rms_eps" in the key store names it. */
static float g_eps;
static int g_dead;
static char g_reason[256];

static void die(const char *why)
{
	g_dead = 1;
	snprintf(g_reason, sizeof(g_reason), "%s", why);
}

#define SHIM_VOID(name, params) \
	V7_ABI void name params { die(#name ": not provided by the oracle shim"); }
#define SHIM_RET(type, name, params, value) \
	V7_ABI type name params { die(#name ": not provided by the oracle shim"); return (type)(value); }
V7G_STUBS_VOID(SHIM_VOID)
V7G_STUBS_RET(SHIM_RET)

V7_ABI void v7s_rmsnorm(float *o, float *x, float *weight, int size)
{
	if (orc_rmsnorm_rows(o, x, weight, 1, size, g_eps, 1) != 0)
		die("v7s_rmsnorm: size % 32 != 0");
}
V7_ABI void v7s_add_inplace(float *x, float *y, int n) { orc_add_inplace(x, y, n, 1); }
V7_ABI void v7s_fused_add_rmsnorm(float *o, float *residual, float *add, float *weight, int dim)
{
	if (orc_fused_add_rmsnorm_rows(o, residual, add, weight, 1, dim, g_eps, 1) != 0)
		die("v7s_fused_add_rmsnorm: dim % 8 != 0");
}
V7_ABI void v7s_rmsnorm_rope_heads(float *buf, int n_heads, int head_dim, float *norm_weight, float *cos_table, float *sin_table, int pos, int rope_max_dim)
{
	/* one token at position pos: the rows entry with tokens = 1 and pos0 = pos */
	if (orc_rmsnorm_rope_rows(buf, 1, n_heads, head_dim, norm_weight, cos_table, sin_table, pos, rope_max_dim, g_eps, 1) != 0)
		die("v7s_rmsnorm_rope_heads: contract violation");
}
V7_ABI void v7d_quantize(char *out_q, float *in_x, float *out_s, int n)
{
	if (orc_quantize_rows((int8_t *)out_q, out_s, in_x, 1, n, 1) != 0)
		die("v7d_quantize: n <= 0");
}
V7_ABI void v7s_rmsnorm_quantize(char *out_q, float *in_x, float *out_s, int n, float *weight)
{
	if (orc_rmsnorm_quantize_rows((int8_t *)out_q, out_s, in_x, weight, 1, n, g_eps, 1) != 0)
		die("v7s_rmsnorm_quantize: n % 64 != 0");
}

V7_ABI void v7d_q8(float *xout, v7_q8_tensor *x, v7_q8_tensor *w, int n, int d)
{
	if (orc_q8_gemv(xout, (const int8_t *)x->q, x->s, (const int8_t *)w->q, w->s, 1, n, d, 16) != 0)
		die("v7d_q8: n % 64 != 0");
}
V7_ABI void v7d_swiglu(float *xout, v7_f32_tensor *x, v7_q8_tensor *gate_w, int n, int d, v7_q8_tensor *up_w)
{
	if (orc_swiglu_f32q8_gemv(xout, x->data, (const int8_t *)gate_w->q, gate_w->s, (const int8_t *)up_w->q, up_w->s, 1, n, d, 0, 16) != 0)
		die("v7d_swiglu: n % 64 != 0");
}
V7_ABI void v7d_swiglu_q8(float *xout, v7_q8_tensor *x, v7_q8_tensor *gate_w, int n, int d, v7_q8_tensor *up_w)
{
	if (orc_swiglu_q8_gemv(xout, (const int8_t *)x->q, x->s, (const int8_t *)gate_w->q, gate_w->s, (const int8_t *)up_w->q, up_w->s, 1, n, d, 16) != 0)
		die("v7d_swiglu_q8: n % 64 != 0");
}

V7_ABI int v7_init(const char *db_path) { return 1; }
V7_ABI int v7_db_load(const char *path) { return 0; }
V7_ABI int v7_db_save(const char *path) { return 0; }
V7_ABI int v7_engine_is_dead(void) { return g_dead; }
V7_ABI const char *v7_get_death_reason(void) { return g_reason; }
V7_ABI const char *v7_get_version(void) { return "v7 oracle shim"; }
V7_ABI int v7_get_console_width(void) { return 80; }
V7_ABI void v7_shutdown(void) {}
V7_ABI void v7s_rope_init(int head_dim, float rope_base) {}
V7_ABI void v7s_set_fused_rope(int pos, int head_dim) {}
V7_ABI void v7s_set_spin(int flag) {}
V7_ABI void v7s_enable_thinking(int on) {}
V7_ABI void v7s_shutdown(void) {}
V7_ABI int v7s_get_num_workers(void) { return 1; }
V7_ABI unsigned long long get_config_was_fixed(void) { return 0; }
V7_ABI void v7_do_fatal(const char *message) { die(message ? message : "v7_do_fatal"); }
V7_ABI void ht_init(void) {}
V7_ABI void ht_destroy(void) {}
V7_ABI int ht_add(const char *key, void *data, unsigned long long data_len, unsigned int persist)
{
	if (key && data && data_len == 4 && strcmp(key, "__sys_rms_eps") == 0) {
		memcpy(&g_eps, data, 4);
		return 1;
	}
	return 0;
}
V7_ABI void *ht_find(const char *key, unsigned long long *out_len)
{
	if (key && strcmp(key, "__sys_rms_eps") == 0) {
		if (out_len)
			*out_len = 4;
		return &g_eps;
	}
	return 0;
}
V7_ABI int v7_db_add(const char *key, const void *data, int len, unsigned int persist) { return ht_add(key, (void *)data, (unsigned long long)len, persist); }
V7_ABI void *v7_db_find(const char *key, unsigned long long *out_len) { return ht_find(key, out_len); }
V7_ABI int db_save(const char *filename) { return 0; }
V7_ABI int db_load(const char *filename) { return 0; }
V7_ABI void db_set_readonly(int flag) {}
V7_ABI int v7sprintf(char *buffer, int buf_size, const char *format, ...)
{
	if (buffer && buf_size > 0)
		buffer[0] = 0;
	return 0;
}
