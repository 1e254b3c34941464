/* CPU oracle for the fused causal convolution.  TEST INFRASTRUCTURE ONLY: used by tests/, by
 * __graft_entry__.smoke() and by bench.py's cpu_baseline / --impl reference leg as the checker and
 * the timed CPU baseline.  Never linked into or called from the product path.
 *
 * Restates, in plain C:
 *   - the reference's fp64 direct causal convolution used to validate cuFFT
 *     (sfFFT src/sffft.cu:376-378):  y[n] = sum_{m<=n} (double)u[m] * (double)k[n-m]
 *   - the reference's seeded generator (src/sffft.cu:308-310): xorshift64 (13, 7, 17) from the
 *     default state 88172645463325252, uniform ((x>>11)+0.5)/2^53, Box-Muller
 *     sqrt(-2 log U1) * cos(2 pi U2) with U1 drawn before U2;
 *   - the reference's input recipe (src/sffft.cu:339-341): u = nrand()*input_scale over B*H*L in
 *     order, then per channel h: a = 1/(4 + L*h/H), k[h,n] = nrand()*exp(-a*n)*sqrt(2a);
 *   - the benchmark configurations' profiles: u ~ N(0,1); k[h,n] = N(0,1)*exp(-decay*n/L) [/sqrt(L)], same stream;
 *   - the same fp64 direct sum for the two filter layouts the reference lists as not yet exposed
 *     (README.md:174): two-sided y[n] = sum_{m<L} u[m] k2[L-1+n-m] (k2 has 2L-1 taps, k2[L-1] is lag 0)
 *     and period-L circular y[n] = sum_{m<L} u[m] kc[(n-m) mod L].  No reference output pins these; the
 *     tests pin them against numpy's fp64 FFT and against the causal sum (a two-sided filter whose
 *     negative lags are zero is the causal filter).
 * The generator stream is pinned by tests/golden/ref_rng.json, produced by compiling the reference's
 * own nrand() (oracle/ref_harness.cu).
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef struct {
  unsigned long long s;
} oracle_rng;

static double urand(oracle_rng* r) {
  r->s ^= r->s << 13;
  r->s ^= r->s >> 7;
  r->s ^= r->s << 17;
  return ((double)(r->s >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}

static double nrand(oracle_rng* r) {
  const double u1 = urand(r);
  const double u2 = urand(r);
  return sqrt(-2 * log(u1)) * cos(2 * M_PI * u2);
}

/* First n normal draws of the stream from `seed` (0 selects the reference default). */
void oracle_nrand_stream(unsigned long long seed, int n, double* out) {
  oracle_rng r = {seed ? seed : 88172645463325252ULL};
  for (int i = 0; i < n; i++) out[i] = nrand(&r);
}

/* Reference recipe (src/sffft.cu:339-341). */
void oracle_gen_reference(unsigned long long seed, int B, int H, int L, double input_scale, float* u, float* k) {
  oracle_rng r = {seed ? seed : 88172645463325252ULL};
  const size_t n = (size_t)B * H * L;
  for (size_t i = 0; i < n; i++) u[i] = (float)(nrand(&r) * input_scale);
  for (int h = 0; h < H; h++) {
    const double a = 1.0 / (4.0 + (double)L * h / H);
    for (int t = 0; t < L; t++) k[(size_t)h * L + t] = (float)(nrand(&r) * exp(-a * t) * sqrt(2 * a));
  }
}

/* Benchmark-configuration profile: k[h,n] = N(0,1) * exp(-decay * n / L) * (sqrt_norm ? 1/sqrt(L) : 1). */
void oracle_gen_profile(unsigned long long seed, int B, int H, int L, double decay, int sqrt_norm, float* u, float* k) {
  oracle_rng r = {seed ? seed : 88172645463325252ULL};
  const size_t n = (size_t)B * H * L;
  const double norm = sqrt_norm ? 1.0 / sqrt((double)L) : 1.0;
  for (size_t i = 0; i < n; i++) u[i] = (float)nrand(&r);
  for (int h = 0; h < H; h++)
    for (int t = 0; t < L; t++) k[(size_t)h * L + t] = (float)(nrand(&r) * exp(-decay * t / L) * norm);
}

static void conv_one(const float* u, const float* k, double* y, int L) {
  for (int n = 0; n < L; n++) {
    double acc = 0;
    for (int m = 0; m <= n; m++) acc += (double)u[m] * (double)k[n - m];
    y[n] = acc;
  }
}

/* fp64 direct causal convolution of the listed sequences (s = b*H + h); y is [nseq][L].
 * threads <= 0 uses every available core. */
void oracle_direct_conv_seqs(const float* u, const float* k, double* y, int B, int H, int L, const long long* seqs,
                             int nseq, int threads) {
  (void)B;
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
#endif
  for (int i = 0; i < nseq; i++) {
    const long long s = seqs[i];
    const int h = (int)(s % H);
    conv_one(u + (size_t)s * L, k + (size_t)h * L, y + (size_t)i * L, L);
  }
}

/* fp64 direct causal convolution of all B*H sequences; y is [B][H][L]. */
void oracle_direct_conv(const float* u, const float* k, double* y, int B, int H, int L, int threads) {
  const long long n = (long long)B * H;
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 4) num_threads(threads)
#endif
  for (long long s = 0; s < n; s++) conv_one(u + (size_t)s * L, k + (size_t)(s % H) * L, y + (size_t)s * L, L);
}

/* Direct sums for one sequence: layout 1 = two-sided (k has 2L-1 taps), 2 = period-L circular. */
static void conv_one_layout(const float* u, const float* k, double* y, int L, int layout) {
  for (int n = 0; n < L; n++) {
    double acc = 0;
    if (layout == 1) {
      for (int m = 0; m < L; m++) acc += (double)u[m] * (double)k[L - 1 + n - m];
    } else {
      for (int m = 0; m < L; m++) acc += (double)u[m] * (double)k[((n - m) % L + L) % L];
    }
    y[n] = acc;
  }
}

/* fp64 direct two-sided (layout 1, k [H][2L-1]) or circular (layout 2, k [H][L]) convolution of the
 * listed sequences (s = b*H + h); y is [nseq][L]. */
void oracle_direct_conv_layout_seqs(const float* u, const float* k, int layout, double* y, int B, int H, int L,
                                    const long long* seqs, int nseq, int threads) {
  (void)B;
  const size_t width = layout == 1 ? (size_t)(2 * L - 1) : (size_t)L;
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
#endif
  for (int i = 0; i < nseq; i++) {
    const long long s = seqs[i];
    const int h = (int)(s % H);
    conv_one_layout(u + (size_t)s * L, k + (size_t)h * width, y + (size_t)i * L, L, layout);
  }
}

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
