/* msabi_shim.c -- test infrastructure: lets Python's ctypes (System V calling
 * convention only) call the library's reference-surface entries, which use the
 * Microsoft x64 convention the reference's loader expects (src/v7_lib.h:40-46).
 * Each shim takes the entry's address (dlsym / ctypes) and its arguments. */
#define V7_ABI __attribute__((ms_abi))

typedef void(V7_ABI *rmsnorm_fn)(float *, float *, float *, int);
typedef void(V7_ABI *add_fn)(float *, float *, int);

void shim_v7s_rmsnorm(void *fn, float *o, float *x, float *w, int size) { ((rmsnorm_fn)fn)(o, x, w, size); }
void shim_v7s_add_inplace(void *fn, float *x, float *y, int n) { ((add_fn)fn)(x, y, n); }

typedef void(V7_ABI *batch4_fn)(const void *);
void shim_q8_batch4(void *fn, const void *args) { ((batch4_fn)fn)(args); }
