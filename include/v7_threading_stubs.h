/* v7_threading_stubs.h -- the 61 reference exports outside the kernel path.
 *
 * v7_load (src/v7_lib.h:585-739) refuses a library that lacks any of its 99
 * names, so these are exported too.  They belong to subsystems this library
 * does not provide (model forward passes, chat/generate, sampler, tokenizer,
 * the fp32-activation matmuls and attention kernels, vision, SectorLogo, KV-cache files,
 * MicroDB compression, the cycle tuner).  Each one marks the engine dead with
 * the reason "<name>: not provided by v7g" (v7_engine_is_dead() = 1, the
 * reference's FATAL contract, src/v7_lib.h:179-184) and returns the value
 * listed here.  Pointer-returning statistics getters return a zeroed block
 * instead of NULL, so hosts that read them unconditionally stay safe.
 *
 * X-macro lists, expanded by the library to define the stubs:
 *   V7G_STUBS_VOID(X)  X(name, (params))
 *   V7G_STUBS_RET(X)   X(return type, name, (params), return value)
 * Declarations follow the reference typedefs at the cited src/v7_lib.h lines.
 */
#ifndef V7_THREADING_STUBS_H
#define V7_THREADING_STUBS_H

#ifdef __cplusplus
extern "C" {
#endif

/* a zeroed block returned by the statistics getters (16 x u64) */
extern unsigned long long v7g_zero_block[16];

#define V7G_STUBS_VOID(X) \
	X(v7d_f32, (float *xout, v7_f32_tensor *x, v7_q8_tensor *w, int n, int d))                                      /* :114 */ \
	X(v7d_fused_f32, (float *xout, v7_f32_tensor *x, v7_q8_tensor *w, int n, int d, float *norm_weights, int is_q)) /* :115 */ \
	X(v7d_attention, (struct v7_run_state *s, struct v7_config *p, int pos, unsigned long long loff, int kv_dim, int kv_mul)) /* :119 */ \
	X(v7d_attention_prefill, (struct v7_run_state *s, struct v7_config *p, float *q_storage, float *att_out_storage, int start_pos, int n_tokens, unsigned long long loff, int kv_dim, int kv_mul)) /* :121 */ \
	X(v7d_memcpy, (void *dst, void *src, int byte_count))                                                         /* :125 */ \
	X(v7d_vit_linear, (float *out, float *in, float *w, float *bias, int n_rows, int M, int K))                   /* :126 */ \
	X(v7s_bicubic_resize, (const unsigned char *src, int src_w, int src_h, unsigned char *dst, int dst_w, int dst_h)) /* :128 */ \
	X(set_prefetch_distance, (int slot, int distance))                                                            /* :289 */ \
	X(set_prefetch_type, (int slot, int type))                                                                    /* :290 */ \
	X(encode, (void *tok, const char *text, int *tokens, int *n_tokens, int max_tokens))                          /* :353 */ \
	X(v7_free_inference, (void))                                                                                  /* :171 */ \
	X(v7_chat, (const char *user_prompt, const char *system_prompt, char *output, int output_len, int reset))    /* :172 */ \
	X(v7_generate, (const char *prompt, char *output, int output_len, int raw_generation))                       /* :175 */ \
	X(v7_generate_image, (const char *user_prompt, const unsigned char *raw_rgb, int img_w, int img_h, char *output, int output_len)) /* :177 */ \
	X(v7_set_sampler_temperature, (float t))                                                                      /* :178 */ \
	X(v7_set_sampler_topp, (float p))                                                                             /* :216 */ \
	X(v7_set_sampler_presence_penalty, (float p))                                                                 /* :217 */ \
	X(v7_set_sampler_topk, (int k))                                                                               /* :218 */ \
	X(v7_set_sampler_seed, (unsigned long long seed))                                                             /* :219 */ \
	X(v7_set_quantize, (int mode))                                                                                /* :220 */ \
	X(v7_set_max_gen, (int cap))                                                                                  /* :221 */ \
	X(v7_set_position, (int pos))                                                                                 /* :223 */ \
	X(v7_get_token_probs, (const int *token_ids, int n, float *out_probs))                                        /* :231 */ \
	X(v7_set_worker_priority, (int priority))                                                                     /* :236 */ \
	X(v7_enable_thinking, (int on))                                                                               /* :237 */ \
	X(v7_encode, (const char *text, int *tokens, int *n_tokens, int max_tokens))                                  /* :240 */ \
	X(v7s_set_caller_hmodule, (void *hmodule))                                                                    /* :299 */ \
	X(v7s_set_vision_embeddings, (float *embeddings, int emb_count, float *ds0, float *ds1, float *ds2))          /* :325 */ \
	X(v7s_vit_forward, (const float *pixels, int grid_h, int grid_w, const void *weights, float *out_main, float *out_ds0, float *out_ds1, float *out_ds2)) /* :351 */ \
	X(v7s_mrope_prepare, (const int *tokens, int n_tokens, int start_pos))                                        /* :256 */ \
	X(v7s_mrope_restore, (void))                                                                                  /* :257 */

#define V7G_STUBS_RET(X) \
	X(int, v7s_sample, (float *logits, int vocab_size, float temperature, float topp, unsigned long long *rng_state, struct v7_probindex *probindex), 0) /* :269 */ \
	X(int, v7s_sectorlogo_eval_script, (const char *key_name), 0)                                                 /* :291 */ \
	X(int, v7_initialize_inference, (void), 0)                                                                    /* :170 */ \
	X(int, v7_chat_image, (const char *user_prompt, const char *system_prompt, const unsigned char *raw_rgb, int img_w, int img_h, char *output, int output_len, int reset), 0) /* :176 */ \
	X(char *, v7_execute_fmt, (char *exe, char *fmt, unsigned long long *argv, int argc), 0)                      /* :187 */ \
	X(const char *, v7s_get_user_prompt, (void), 0)                                                               /* :191 */ \
	X(int, save_kv_cache, (const char *filename), 0)                                                              /* :205 */ \
	X(int, load_kv_cache, (const char *filename), 0)                                                              /* :206 */ \
	X(int, v7_set_streaming, (int enable, int num_sinks, int window_size), -1)                                    /* :215 */ \
	X(int, v7_get_position, (void), 0)                                                                            /* :222 */ \
	X(int, v7_get_think_mode_active, (void), 0)                                                                   /* :226 */ \
	X(int, v7_get_gen_count, (void), 0)                                                                           /* :230 */ \
	X(unsigned long long *, v7_get_generation_statistic, (void), v7g_zero_block)                                 /* :241 */ \
	X(unsigned long long *, v7_get_best_fitness, (void), v7g_zero_block)                                         /* :247 */ \
	X(unsigned long long *, v7_get_pool_fitness, (void), v7g_zero_block)                                         /* :248 */ \
	X(int, v7_get_active_shape_count, (void), 0)                                                                  /* :249 */ \
	X(struct inference_context *, v7_get_internal_inference_ctx, (void), 0)                                       /* :254 */ \
	X(int, v7s_sectorlogo_on_token, (struct inference_context *ctx, int token_id, int position, int *out_token, float *temperature, float *topp), 0) /* :297 */ \
	X(int, v7s_sectorlogo_interp, (const char *script), 0)                                                        /* :298 */ \
	X(char *, v7_execute, (const char *exe, const char *parameter1, const char *parameter2, const char *parameter3), 0) /* :301 */ \
	X(char *, v7s_readfile, (const char *path), 0)                                                                /* :320 */ \
	X(int, v7s_writefile, (const char *path, char *text, int append), 0)                                          /* :321 */ \
	X(int, v7s_vit_encode_callback, (const unsigned char *raw_rgb, int img_w, int img_h, float **out_emb, int *out_count, float **out_ds0, float **out_ds1, float **out_ds2), 1) /* :348 */ \
	X(unsigned long long *, v7s_get_generation_statistic, (void), v7g_zero_block)                                /* :342 */ \
	X(float *, forward_f32, (void *transformer, int token, int pos), 0)                                          /* :355 */ \
	X(float *, forward_q8, (void *transformer, int token, int pos), 0)                                           /* :356 */ \
	X(float *, prefill_forward_f32, (void *transformer, int *tokens, int n_tokens, int start_pos), 0)            /* :357 */ \
	X(float *, prefill_forward_q8, (void *transformer, int *tokens, int n_tokens, int start_pos), 0)             /* :358 */ \
	X(unsigned long long, mdb_compress, (const void *src, unsigned long long src_len, void *dst), 0)              /* :136 */ \
	X(unsigned long long, mdb_decompress, (void *src, unsigned long long src_len, void *dst, unsigned long long max_dst), 0) /* :137 */

#define V7G_DECLARE_VOID(name, params) V7_ABI void name params;
#define V7G_DECLARE_RET(type, name, params, value) V7_ABI type name params;
V7G_STUBS_VOID(V7G_DECLARE_VOID)
V7G_STUBS_RET(V7G_DECLARE_RET)
#undef V7G_DECLARE_VOID
#undef V7G_DECLARE_RET

#ifdef __cplusplus
}
#endif
#endif
