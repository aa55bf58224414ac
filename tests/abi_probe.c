/* abi_probe.c -- drives libv7_threading.so the way the reference's host
 * loader does (dlopen + dlsym, Microsoft x64 calling convention,
 * src/v7_lib.h:585-739) and prints one line per check.  Built and run by
 * tests/test_abi_exports.py (CPU: only host-side behaviour) and
 * tests/test_ref_harness_gpu.py (GPU: the hot-path entries on host and device
 * pointers).
 *
 * usage: abi_probe <lib> <names-file> [gpu]
 */
#include <dlfcn.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "v7_threading.h"

#define RESOLVE(T, name) T p_##name = (T)dlsym(h, #name)

typedef int(V7_ABI *init_fn)(const char *);
typedef int(V7_ABI *dead_fn)(void);
typedef const char *(V7_ABI *reason_fn)(void);
typedef int(V7_ABI *ht_add_fn)(const char *, void *, unsigned long long, unsigned int);
typedef void *(V7_ABI *ht_find_fn)(const char *, unsigned long long *);
typedef void(V7_ABI *rmsnorm_fn)(float *, float *, float *, int);
typedef void(V7_ABI *add_fn)(float *, float *, int);
typedef void(V7_ABI *chat_fn)(const char *, const char *, char *, int, int);
typedef int(V7_ABI *save_fn)(const char *);
typedef int *int_ptr;
typedef void(V7_ABI *rope_init_fn)(int, float);
typedef void(V7_ABI *rope_only_fn)(float *, int, int, float *, float *, int, int);
typedef void(V7_ABI *rope_heads_fn)(float *, int, int, float *, float *, float *, int, int);
typedef void(V7_ABI *qk_fork_fn)(const v7_qk_fork_args *);
typedef int (*get_tables_fn)(const float **, const float **, int *);

static int failures = 0;
#define CHECK(cond, msg)                                           \
	do {                                                           \
		if (cond)                                                  \
			printf("ok   %s\n", msg);                              \
		else {                                                     \
			printf("FAIL %s\n", msg);                              \
			failures++;                                            \
		}                                                          \
	} while (0)

int main(int argc, char **argv)
{
	if (argc < 3) {
		fprintf(stderr, "usage: %s <lib> <names-file> [gpu]\n", argv[0]);
		return 2;
	}
	int gpu = argc > 3 && strcmp(argv[3], "gpu") == 0;
	void *h = dlopen(argv[1], RTLD_NOW | RTLD_LOCAL);
	if (!h) {
		printf("FAIL dlopen: %s\n", dlerror());
		return 1;
	}
	/* every name the reference's loader resolves */
	FILE *f = fopen(argv[2], "r");
	char name[256];
	int missing = 0, total = 0;
	while (f && fscanf(f, "%255s", name) == 1) {
		total++;
		if (!dlsym(h, name)) {
			printf("FAIL missing export %s\n", name);
			missing++;
		}
	}
	if (f)
		fclose(f);
	printf("%s %d/%d loader names resolved\n", missing ? "FAIL" : "ok  ", total - missing, total);
	failures += missing;

	RESOLVE(init_fn, v7_init);
	RESOLVE(dead_fn, v7_engine_is_dead);
	RESOLVE(reason_fn, v7_get_death_reason);
	RESOLVE(ht_add_fn, ht_add);
	RESOLVE(ht_find_fn, ht_find);
	RESOLVE(rmsnorm_fn, v7s_rmsnorm);
	RESOLVE(add_fn, v7s_add_inplace);
	RESOLVE(chat_fn, v7_chat);
	RESOLVE(save_fn, db_save);
	RESOLVE(init_fn, db_load);
	RESOLVE(rope_init_fn, v7s_rope_init);
	RESOLVE(rope_only_fn, v7s_rope_only_heads);
	RESOLVE(rope_heads_fn, v7s_rmsnorm_rope_heads);
	RESOLVE(qk_fork_fn, v7s_qk_fork_heads);
	RESOLVE(get_tables_fn, v7g_get_rope_tables);
	int_ptr p_cpu_features_ok = (int_ptr)dlsym(h, "cpu_features_ok");

	CHECK(p_v7_init(NULL) == 1, "v7_init(NULL) succeeds");
	CHECK(!p_v7_engine_is_dead(), "engine alive after init");
	CHECK(p_v7_init("/nonexistent/v7.db") == 0 && p_v7_engine_is_dead(), "v7_init of a missing file fails and kills the engine");
	CHECK(p_v7_init(NULL) == 1 && !p_v7_engine_is_dead(), "v7_init(NULL) revives");
	CHECK(p_cpu_features_ok && *p_cpu_features_ok == 1, "cpu_features_ok data word is 1");

	float eps = 1e-6f;
	CHECK(p_ht_add("__sys_rms_eps", &eps, 4, 0) == 1, "ht_add(__sys_rms_eps)");
	unsigned long long len = 0;
	float *pe = (float *)p_ht_find("__sys_rms_eps", &len);
	CHECK(pe && len == 4 && *pe == eps, "ht_find(__sys_rms_eps) returns the kernels' eps");
	int v = 42;
	CHECK(p_ht_add("user_key", &v, 4, 0) == 1, "ht_add(user_key)");
	const char *db = "/tmp/v7g_abi_probe.db";
	CHECK(p_db_save(db) == 1, "db_save");
	eps = 0.0f;
	p_ht_add("__sys_rms_eps", &eps, 4, 0);
	CHECK(p_v7_init(db) == 1, "v7_init(saved store)");
	pe = (float *)p_ht_find("__sys_rms_eps", &len);
	int *pv = (int *)p_ht_find("user_key", &len);
	CHECK(pe && *pe == 1e-6f && pv && *pv == 42 && len == 4, "store round trip restores keys and eps");
	remove(db);

	char out[16];
	p_v7_chat("hi", NULL, out, sizeof(out), 1);
	CHECK(p_v7_engine_is_dead() && strstr(p_v7_get_death_reason(), "v7_chat") != NULL, "out-of-scope export marks the engine dead with its name");
	p_v7_init(NULL);

	float x[64], w[64], o[64];
	for (int i = 0; i < 64; ++i) {
		x[i] = (float)(i % 7) - 3.0f;
		w[i] = 1.0f;
		o[i] = -99.0f;
	}
	p_v7s_rmsnorm(o, x, w, 48);
	CHECK(p_v7_engine_is_dead() && strstr(p_v7_get_death_reason(), "size") && o[0] == -99.0f, "v7s_rmsnorm rejects size % 32 != 0 without writing");
	p_v7_init(NULL);

	/* v7s_rope_init reads its parameters from the key store; a missing key is
	   fatal in the reference (ht_find_or_fatal) */
	p_v7s_rope_init(128, 1e6f);
	CHECK(p_v7_engine_is_dead() && strstr(p_v7_get_death_reason(), "__sys_rope_base"), "v7s_rope_init without __sys_rope_base kills the engine naming the key");
	p_v7_init(NULL);
	float rope_base = 1e6f;
	int rope_type = 0;
	p_ht_add("__sys_rope_base", &rope_base, 4, 0);
	p_ht_add("__sys_rope_type", &rope_type, 4, 0);

	if (!gpu) {
		p_v7s_rope_init(128, 0.0f);
		CHECK(p_v7_engine_is_dead() && strstr(p_v7_get_death_reason(), "device"), "v7s_rope_init without a GPU reports death");
		p_v7_init(NULL);
		/* no device here: a valid call must fail cleanly, not crash */
		p_v7s_rmsnorm(o, x, w, 64);
		CHECK(p_v7_engine_is_dead() && o[0] == -99.0f, "v7s_rmsnorm without a GPU reports death and leaves outputs");
	} else {
		eps = 1e-6f;
		p_ht_add("__sys_rms_eps", &eps, 4, 0);
		p_v7s_rmsnorm(o, x, w, 64);
		double ss = 0;
		for (int i = 0; i < 64; ++i)
			ss += (double)x[i] * x[i];
		double sc = 1.0 / sqrt(ss / 64 + 1e-6);
		int good = !p_v7_engine_is_dead();
		for (int i = 0; i < 64; ++i)
			good = good && fabs(o[i] - x[i] * sc) < 1e-5;
		CHECK(good, "v7s_rmsnorm on host pointers computes on the GPU");
		float y[64];
		for (int i = 0; i < 64; ++i)
			y[i] = 0.5f;
		p_v7s_add_inplace(x, y, 64);
		CHECK(!p_v7_engine_is_dead() && x[1] == -1.5f && x[3] == 0.5f, "v7s_add_inplace on host pointers");

		/* rope family: 4 heads of 64 at position 5, tables of rows of 32 */
		enum { H = 4, D = 64, HALF = 32, POS = 5 };
		static float buf[H * D], a1[H * D], a2[H * D], a3[H * D], wn[D], ct[(POS + 1) * HALF], st[(POS + 1) * HALF];
		for (int i = 0; i < H * D; ++i)
			buf[i] = (float)((i * 37) % 23) / 7.0f - 1.5f;
		for (int i = 0; i < D; ++i)
			wn[i] = 1.0f + (float)(i % 5) / 10.0f;
		for (int i = 0; i < (POS + 1) * HALF; ++i) {
			ct[i] = cosf(0.01f * (float)i);
			st[i] = sinf(0.01f * (float)i);
		}
		memcpy(a1, buf, sizeof(buf));
		p_v7s_rope_only_heads(a1, H, D, ct, st, POS, HALF);
		good = !p_v7_engine_is_dead();
		for (int hh = 0; hh < H; ++hh)
			for (int j = 0; j < HALF; ++j) {
				float lo = buf[hh * D + j], hi = buf[hh * D + HALF + j], c = ct[POS * HALF + j], sn = st[POS * HALF + j];
				float lc = lo * c, ls = lo * sn;
				good = good && a1[hh * D + j] == fmaf(-hi, sn, lc) && a1[hh * D + HALF + j] == fmaf(hi, c, ls);
			}
		CHECK(good, "v7s_rope_only_heads on host pointers: exact rotation");
		memcpy(a1, buf, sizeof(buf));
		p_v7s_rope_only_heads(a1, H, D, ct, st, 0, HALF);
		CHECK(!p_v7_engine_is_dead() && memcmp(a1, buf, sizeof(buf)) == 0, "v7s_rope_only_heads at position 0 is the identity");

		memcpy(a2, buf, sizeof(buf));
		memcpy(a3, buf, sizeof(buf));
		p_v7s_rmsnorm_rope_heads(a2, H, D, wn, ct, st, POS, HALF);
		v7_qk_fork_args qa = { a3, wn, ct + POS * HALF, st + POS * HALF, D, H, POS, 0 };
		p_v7s_qk_fork_heads(&qa);
		CHECK(!p_v7_engine_is_dead() && memcmp(a2, a3, sizeof(buf)) == 0, "v7s_qk_fork_heads equals v7s_rmsnorm_rope_heads");

		p_v7s_rope_init(D, 0.0f);
		const float *dc = NULL, *ds = NULL;
		int half = 0;
		CHECK(!p_v7_engine_is_dead() && p_v7g_get_rope_tables(&dc, &ds, &half) == 0 && dc && ds && half == HALF, "v7s_rope_init builds device tables from the key store");
		/* the engine's call: host heads, the library's device tables */
		memcpy(a2, buf, sizeof(buf));
		p_v7s_rmsnorm_rope_heads(a2, H, D, wn, (float *)dc, (float *)ds, POS, HALF);
		CHECK(!p_v7_engine_is_dead(), "v7s_rmsnorm_rope_heads with host heads and device tables");
		FILE *rf = getenv("V7G_PROBE_OUT") ? fopen(getenv("V7G_PROBE_OUT"), "wb") : NULL;
		if (rf) {
			fwrite(buf, sizeof(float), H * D, rf);
			fwrite(wn, sizeof(float), D, rf);
			fwrite(a2, sizeof(float), H * D, rf);
			fclose(rf);
		}
	}
	printf("%s\n", failures ? "PROBE FAILED" : "PROBE PASSED");
	return failures ? 1 : 0;
}
