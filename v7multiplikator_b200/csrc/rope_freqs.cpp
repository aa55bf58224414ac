// rope_freqs.cpp -- the RoPE frequencies freq_j, j < half, on the host.
//
// The reference computes them once per table build on the x87 unit with
// control word 0x037F (extended precision, round to nearest, exceptions
// masked) and stores each as a double (fused_f32_kernel.inc:117-256):
//   plain:  freq_j = base^(-j/half): -j/half times log2(base) by fyl2x, the
//           integer part by frndint, 2^fraction by f2xm1 + 1, scaled back by
//           fscale (:120-137);
//   llama3: inv = that value; wavelen = 2*pi / inv; inv is divided by
//           `factor` when wavelen exceeds the low-frequency wavelength, and
//           blended with the smooth factor in the medium band (:186-256).
// Intermediates the reference keeps in x87 registers stay at extended
// precision here (long double is that 80-bit format on x86-64, and its
// arithmetic is x87 arithmetic); those it stores as doubles are rounded to
// double at the same points.  The table entries are then computed on the
// device (rope_tables.cu).  Half a KB of doubles: no reason to move this part
// off the host.
#include <cstring>

#include "internal.h"

namespace {

constexpr unsigned short kCwExtendedNearest = 0x037F;
constexpr int kMaxHalf = 256;
// 2*pi as the double the reference loads (fused_f32_kernel.inc:65-66)
constexpr double kTwoPi = 6.28318530717958647692;

struct X87Mode {
	unsigned short saved;
	X87Mode()
	{
		__asm__ __volatile__("fnstcw %0" : "=m"(saved));
		unsigned short cw = kCwExtendedNearest;
		__asm__ __volatile__("fldcw %0" : : "m"(cw));
	}
	~X87Mode() { __asm__ __volatile__("fldcw %0" : : "m"(saved)); }
};

long double log2_times(long double x, long double y) // y * log2(x)
{
	long double r;
	__asm__("fyl2x" : "=t"(r) : "0"(x), "u"(y) : "st(1)");
	return r;
}

long double round_int(long double x)
{
	long double r;
	__asm__("frndint" : "=t"(r) : "0"(x));
	return r;
}

long double exp2_minus_one(long double x) // |x| <= 1
{
	long double r;
	__asm__("f2xm1" : "=t"(r) : "0"(x));
	return r;
}

long double scale_pow2(long double x, long double n) // x * 2^trunc(n)
{
	long double r;
	__asm__("fscale" : "=t"(r) : "0"(x), "u"(n));
	return r;
}

long double inv_freq(float base, int j, int half)
{
	const long double t = -((long double)j / (long double)half);
	const long double y = log2_times((long double)base, t);
	const long double n = round_int(y);
	return scale_pow2(exp2_minus_one(y - n) + 1.0L, n);
}

} // namespace

extern "C" int v7g_rope_freqs(double *freqs, int half, float base, int scaling, float factor, float high_freq_factor, float low_freq_factor, int orig_max_pos)
{
	using namespace v7g;
	if (!freqs || half <= 0 || half > kMaxHalf)
		return set_error(V7G_ERR_ARG, "v7g_rope_freqs: need freqs != NULL and 0 < half <= %d", kMaxHalf);
	if (scaling != 0 && scaling != 1)
		return set_error(V7G_ERR_ARG, "v7g_rope_freqs: scaling %d is neither 0 (none) nor 1 (llama3)", scaling);
	X87Mode mode;
	if (scaling == 0) {
		for (int j = 0; j < half; ++j)
			freqs[j] = (double)inv_freq(base, j, half);
		return clear_error();
	}
	const double f = factor, hi = high_freq_factor, lo = low_freq_factor, old_ctx = (double)orig_max_pos;
	const double low_wl = (double)((long double)old_ctx / (long double)lo);
	const double high_wl = (double)((long double)old_ctx / (long double)hi);
	for (int j = 0; j < half; ++j) {
		const long double inv80 = inv_freq(base, j, half);
		const double inv = (double)inv80;
		const double wavelen = (double)((long double)kTwoPi / inv80);
		const double ifl = low_wl < wavelen ? (double)((long double)inv / (long double)f) : inv;
		const long double num = (long double)old_ctx / (long double)wavelen - (long double)lo;
		const double smooth = (double)(num / ((long double)hi - (long double)lo));
		const long double blend = (1.0L - (long double)smooth) * ((long double)ifl / (long double)f) + (long double)smooth * (long double)ifl;
		const double smoothed = (double)blend;
		const bool medium = (high_wl < wavelen && low_wl >= wavelen) || high_wl == wavelen;
		freqs[j] = medium ? smoothed : ifl;
	}
	return clear_error();
}
