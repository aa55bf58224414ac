// gen_golden.cpp -- writes the outputs of the reference's own C reference
// kernels (tools/kt_utils.h) for the cases its validators run, so the oracle
// and the GPU kernels can be checked against them without the reference tree.
//
// Compiled and run by make_golden.py against the reference's headers; the
// inputs are regenerated exactly as the validators do (srand(seed) + glibc
// rand(), tools/kt_utils.h:812-816, :953-972, :1001-1005, :1051-1057,
// :139-191), so only outputs are stored.
//
// Output: a stream of records on stdout
//   u32 name_len, name bytes, u32 kind (0 = float32, 1 = int8), u64 count, data
#include "v7_lib.h"
#include "kt_utils.h"

#include <cstdint>
#include <cstdio>
#include <string>
#include <vector>

static void emit(const std::string &name, const void *data, uint32_t kind, uint64_t count)
{
	uint32_t nl = (uint32_t)name.size();
	fwrite(&nl, 4, 1, stdout);
	fwrite(name.data(), 1, nl, stdout);
	fwrite(&kind, 4, 1, stdout);
	fwrite(&count, 8, 1, stdout);
	fwrite(data, kind == 0 ? 4 : 1, count, stdout);
}

static float eps_default = 1e-6f;

int main()
{
	const int seeds[] = {12345, 67890};
	// v_rmsnorm_validate.cpp:51-61 sizes (repeats dropped), section 1
	const int rms_sizes[] = {64, 128, 256, 1024, 2048, 3072, 8192};
	for (int size : rms_sizes)
		for (int seed : seeds) {
			std::vector<float> x(size), w(size), o(size);
			srand(seed);
			for (int i = 0; i < size; i++)
				x[i] = -1.0f + (float)(rand() % 2001) / 1000.0f;
			for (int i = 0; i < size; i++)
				w[i] = 0.5f + (float)(rand() % 1001) / 1000.0f;
			v7s_rmsnorm_c_ref(o.data(), x.data(), w.data(), size, eps_default);
			emit("rmsnorm/" + std::to_string(size) + "/" + std::to_string(seed), o.data(), 0, size);
		}
	// v_rmsnorm_validate.cpp:87-101 sizes, section 4
	const int add_sizes[] = {8, 16, 24, 48, 64, 128, 256, 1024, 2048, 3072, 8192};
	for (int dim : add_sizes)
		for (int seed : seeds) {
			std::vector<float> r(dim), a(dim), w(dim), o(dim);
			srand(seed);
			for (int i = 0; i < dim; i++)
				r[i] = -1.0f + (float)(rand() % 2001) / 1000.0f;
			for (int i = 0; i < dim; i++)
				a[i] = -1.0f + (float)(rand() % 2001) / 1000.0f;
			for (int i = 0; i < dim; i++)
				w[i] = 0.5f + (float)(rand() % 1001) / 1000.0f;
			v7s_fused_add_rmsnorm_c_ref(o.data(), r.data(), a.data(), w.data(), dim, eps_default);
			emit("add_rmsnorm/" + std::to_string(dim) + "/" + std::to_string(seed), o.data(), 0, dim);
			emit("add_rmsnorm_res/" + std::to_string(dim) + "/" + std::to_string(seed), r.data(), 0, dim);
		}
	// v_rmsnorm_validate.cpp:67-83, section 3 (tables built as in kt_utils.h:953-972)
	struct RopeCase {
		int n_heads, head_dim, pos, rope_max_dim;
		float eps;
	};
	const RopeCase rope[] = {{1, 64, 0, 64, 1e-6f},   {1, 64, 7, 64, 1e-6f},    {4, 64, 0, 64, 1e-6f},    {4, 64, 31, 64, 1e-6f},
	                         {8, 64, 7, 64, 1e-6f},   {8, 128, 0, 128, 1e-6f},  {16, 64, 0, 64, 1e-6f},   {16, 64, 31, 64, 1e-6f},
	                         {32, 64, 7, 64, 1e-6f},  {32, 128, 0, 128, 1e-6f}, {40, 64, 31, 64, 1e-6f},  {40, 128, 7, 128, 1e-6f},
	                         {32, 64, 0, 64, 1e-5f},  {32, 64, 31, 64, 1e-5f},  {8, 64, 7, 64, 1e-5f}};
	for (const RopeCase &c : rope)
		for (int seed : seeds) {
			int n = c.n_heads * c.head_dim;
			std::vector<float> buf(n), w(c.head_dim), ct((size_t)(c.pos + 1) * c.rope_max_dim), st(ct.size());
			srand(seed);
			for (int i = 0; i < n; i++)
				buf[i] = -1.0f + (float)(rand() % 2001) / 1000.0f;
			for (int i = 0; i < c.head_dim; i++)
				w[i] = 0.5f + (float)(rand() % 1001) / 1000.0f;
			int half = c.head_dim / 2;
			for (int p = 0; p <= c.pos; p++) {
				size_t base = (size_t)p * c.rope_max_dim;
				for (int j = 0; j < half; j++) {
					float theta = powf(10000.0f, -2.0f * j / (float)c.head_dim);
					ct[base + j] = cosf(p * theta);
					st[base + j] = sinf(p * theta);
				}
				for (int j = half; j < c.rope_max_dim; j++) {
					ct[base + j] = 0.0f;
					st[base + j] = 0.0f;
				}
			}
			std::string key = std::to_string(c.n_heads) + "x" + std::to_string(c.head_dim) + "/" + std::to_string(c.pos) + "/" +
			                  std::to_string(c.rope_max_dim) + "/" + (c.eps == 1e-5f ? "1e-5" : "1e-6") + "/" + std::to_string(seed);
			emit("rope_cos/" + key, ct.data(), 0, ct.size());
			emit("rope_sin/" + key, st.data(), 0, st.size());
			v7s_rmsnorm_rope_heads_c_ref(buf.data(), c.n_heads, c.head_dim, w.data(), ct.data(), st.data(), c.pos, c.rope_max_dim, c.eps);
			emit("rope/" + key, buf.data(), 0, n);
		}
	// v_add_inplace_validate.cpp:21-22
	const int add_n[] = {32, 64, 96, 128, 160, 1024, 2048};
	for (int n : add_n)
		for (int seed : seeds) {
			std::vector<float> x(n), y(n);
			srand(seed);
			for (int i = 0; i < n; i++)
				x[i] = -10.0f + (float)(rand() % 20001) / 1000.0f;
			for (int i = 0; i < n; i++)
				y[i] = -10.0f + (float)(rand() % 20001) / 1000.0f;
			v7s_add_inplace_c_ref(x.data(), y.data(), n);
			emit("add_inplace/" + std::to_string(n) + "/" + std::to_string(seed), x.data(), 0, n);
		}
	// v_quantize_validate.cpp:14-15, 7 patterns (kt_utils.h:139-191)
	const int q_sizes[] = {64, 256, 1024, 4096, 8192, 65536};
	const int q_seeds[] = {12345, 67890, 11111};
	for (int pat = 0; pat < KTPAT_COUNT; ++pat)
		for (int n : q_sizes)
			for (int seed : q_seeds) {
				std::vector<float> x(n), s((n + 63) / 64);
				std::vector<char> q(n);
				kt_init_quantize_pattern(x.data(), n, seed, pat);
				kt_quantize_c_ref(q.data(), x.data(), s.data(), n);
				std::string key = std::to_string(pat) + "/" + std::to_string(n) + "/" + std::to_string(seed);
				emit("quant_codes/" + key, q.data(), 1, n);
				emit("quant_scales/" + key, s.data(), 0, s.size());
			}
	return 0;
}
