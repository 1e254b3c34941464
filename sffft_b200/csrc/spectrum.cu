// Filter-spectrum preparation: Kf[h][p] = sum_{n<L} k[h][n] * exp(-2*pi*i*n*f(p)/N) in fp32, written in
// the plan's digit order (position p = k0*R1*R2 + k1*R2 + k2 holds frequency f = k0 + R0*k1 + R0*R1*k2).
//
// Replaces the reference's host zero-padding + cufftExecC2C + permuteK (sfFFT src/sffft.cu:342-344,
// 365, 283-288, 384) with one kernel launch per digit that works in place in the caller's Kf buffer:
// stage j loads whole length-R_j vectors of a channel into shared memory, does a direct DFT with an
// exact twiddle table (sincospif of a reduced rational argument), applies the four-step twiddle
// w_N^(R0..R_{j-1} * inner * k_j) (the exponent of src/sffft.cu:106-113, unscaled), and writes the
// vectors back.  Stage 0 reads the real filter (fp32 or bf16) directly and lays it out over the N = 2L
// taps of the circular filter kw that the fused kernel applies to the zero-padded input:
//   causal     k [H][L]:     kw[n] = k[n] for n < L, 0 above (the reference's zero padding);
//   two-sided  k [H][2L-1]:  kw[n] = k[L-1+n] for n < L, kw[L] = 0, kw[N-j] = k[L-1-j] for 0 < j < L,
//                            so y[n] = sum_{m<L} u[m] k[L-1+n-m] (k[L-1] is lag 0);
//   circular   k [H][L]:     kw[n] = k[n mod L], so y[n] = sum_{m<L} u[m] k[(n-m) mod L] (period L).
// The input is zero-padded to N in every case, so lags n - m in (-L, L) never alias; the reference
// exposes only the causal form (README.md:174 lists non-causal and circular convolution as missing).
// Like the reference's prep it runs once per channel and plan, outside the timed convolution.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "spectrum.h"

#include "../../include/sffft.h"

namespace sffft {

struct SpecStage {
  int N, L, R, stride, pre;   // digit radix, stride of the digit, product of the radices before it
  int layout;                 // filter layout of stage 0 (SFFFT_FILTER_*)
  long long kpitch, koff;     // stage 0: element offset of channel h's row is h * kpitch + koff
  int vec_per_cta;            // vectors handled by one CTA
  int twiddle;                // apply the inter-stage twiddle after this digit (not the last digit)
};

__device__ __forceinline__ float k_to_float(float v) { return v; }
__device__ __forceinline__ float k_to_float(__nv_bfloat16 v) { return __bfloat162float(v); }

// Where stage 0 takes its input from: the buffer itself (later stages), a real row per channel placed
// by a filter layout (kLayoutFull: all N samples, the standalone forward FFT), or the conjugated
// Hermitian extension of a half spectrum [N/2 + 1] (the standalone inverse FFT, computed as
// conj(DFT(conj(X))) / N).
enum { kSrcInPlace = 0, kSrcReal = 1, kSrcHermitian = 2 };
constexpr int kLayoutFull = 3;


template <class TK, int SRC>
__global__ void __launch_bounds__(256) spectrum_stage_kernel(float2* __restrict__ Kf, const TK* __restrict__ k, SpecStage st) {
  extern __shared__ float2 sbuf[];
  float2* tab = sbuf;                 // w_R^q, q in [0, R)
  float2* x = sbuf + st.R;            // vec_per_cta vectors of R complex values
  const int R = st.R, VB = st.vec_per_cta, N = st.N;
  const int vec_per_ch = N / R, cta_per_ch = vec_per_ch / VB;
  const int h = blockIdx.x / cta_per_ch, v0 = (blockIdx.x % cta_per_ch) * VB;
  float2* Kh = Kf + (size_t)h * N;

  for (int q = threadIdx.x; q < R; q += blockDim.x) {
    float s, c;
    sincospif(-2.0f * (float)q / (float)R, &s, &c);
    tab[q] = make_float2(c, s);
  }
  for (int i = threadIdx.x; i < VB * R; i += blockDim.x) {
    const int vl = i / R, d = i - vl * R, v = v0 + vl;
    const int outer = v / st.stride, inner = v - outer * st.stride;
    const int p = outer * R * st.stride + d * st.stride + inner;
    float2 val;
    if constexpr (SRC == kSrcHermitian) {
      const float2* X = reinterpret_cast<const float2*>(k) + (size_t)h * (N / 2 + 1);
      if (p <= N / 2) {
        const float2 xv = X[p];
        val = make_float2(xv.x, (p == 0 || p == N / 2) ? 0.f : -xv.y);
      } else {
        val = X[N - p];
      }
    } else if constexpr (SRC == kSrcReal) {
      const int L = st.L;
      int col = -1;   // column of the filter row that lands on tap p, or -1 for a zero tap
      if (st.layout == SFFFT_FILTER_TWO_SIDED) {
        col = p < L ? L - 1 + p : (p > L ? p - L - 1 : -1);   // tap N - j (0 < j < L) holds lag -j
      } else if (st.layout == SFFFT_FILTER_CIRCULAR) {
        col = p & (L - 1);
      } else if (st.layout == kLayoutFull) {
        col = p;
      } else if (st.layout == kLayoutSegment) {
        col = p < L ? L + p : p - L;
      } else {
        col = p < L ? p : -1;
      }
      const long long ix = st.koff + col;
      val = make_float2(col >= 0 && ix >= 0 ? k_to_float(k[h * st.kpitch + ix]) : 0.f, 0.f);
    } else {
      val = Kh[p];
    }
    x[i] = val;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < VB * R; i += blockDim.x) {
    const int vl = i / R, kk = i - vl * R, v = v0 + vl;
    const float2* xv = x + vl * R;
    float re = 0.f, im = 0.f;
    for (int d = 0; d < R; d++) {
      const float2 w = tab[(d * kk) & (R - 1)], a = xv[d];
      re = fmaf(a.x, w.x, fmaf(-a.y, w.y, re));
      im = fmaf(a.x, w.y, fmaf(a.y, w.x, im));
    }
    const int outer = v / st.stride, inner = v - outer * st.stride;
    if (st.twiddle) {
      int e = (int)(((long long)st.pre * inner * kk) & (N - 1));
      if (e > N / 2) e -= N;
      float s, c;
      sincospif(-2.0f * (float)e / (float)N, &s, &c);
      const float nr = re * c - im * s;
      im = re * s + im * c;
      re = nr;
    }
    Kh[outer * R * st.stride + kk * st.stride + inner] = make_float2(re, im);
  }
}

// Natural order out of the digit-order buffer W [rows][N]: the forward FFT writes the half spectrum
// X[f] = W[pos(f)], f <= N/2; the inverse writes x[n] = Re W[pos(n)] / N (W = DFT(conj(Xfull)), whose
// conjugate has the same real part).  pos(f) = k0*R1*R2 + k1*R2 + k2 for f = k0 + R0*k1 + R0*R1*k2.
template <bool INV>
__global__ void __launch_bounds__(256) fft_gather_kernel(const float2* __restrict__ W, void* __restrict__ out, int rows,
                                                         int R0, int R1, int R2) {
  const int N = R0 * R1 * R2, width = INV ? N : N / 2 + 1;
  const long long total = (long long)rows * width;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / width;
    const int f = (int)(i - r * width);
    const int k0 = f % R0, k1 = (f / R0) % R1, k2 = f / (R0 * R1);
    const float2 v = W[r * N + (k0 * R1 + k1) * R2 + k2];
    if constexpr (INV) reinterpret_cast<float*>(out)[i] = v.x * (1.0f / (float)N);
    else reinterpret_cast<float2*>(out)[i] = v;
  }
}

// Runs the digit stages for radices R[0..S-1] over H channels of a filter for length L = N/2 in the
// given layout.  k_bf16: the filter holds bf16 values instead of fp32.  hermitian: k is a half spectrum
// [H][N/2 + 1] of float2 for the inverse FFT (layout and k_bf16 unused).  kpitch / koff: the filter row of
// channel h starts at element h * kpitch + koff (kpitch < 0: the layout's own row width, koff = 0).
cudaError_t launch_spectrum(float2* Kf, const void* k, bool k_bf16, int layout, int H, const int* R, int S,
                            cudaStream_t stream, bool hermitian, long long kpitch, long long koff) {
  int N = 1;
  for (int j = 0; j < S; j++) N *= R[j];
  if (kpitch < 0) {
    kpitch = layout == SFFFT_FILTER_TWO_SIDED ? N - 1 : (layout == kLayoutFull ? N : N / 2);
    koff = 0;
  }
  int stride = N, pre = 1;
  for (int j = 0; j < S; j++) {
    stride /= R[j];
    SpecStage st;
    st.N = N; st.L = N / 2; st.layout = layout; st.kpitch = kpitch; st.koff = koff; st.R = R[j]; st.stride = stride; st.pre = pre; st.twiddle = (j + 1 < S);
    const int vec_per_ch = N / R[j];
    st.vec_per_cta = vec_per_ch < 2048 / R[j] ? vec_per_ch : 2048 / R[j];
    const int grid = H * (vec_per_ch / st.vec_per_cta);
    const size_t smem = (size_t)(st.R + st.vec_per_cta * st.R) * sizeof(float2);
    if (j == 0 && hermitian) {
      spectrum_stage_kernel<float2, kSrcHermitian><<<grid, 256, smem, stream>>>(Kf, (const float2*)k, st);
    } else if (j == 0) {
      if (k_bf16) spectrum_stage_kernel<__nv_bfloat16, kSrcReal><<<grid, 256, smem, stream>>>(Kf, (const __nv_bfloat16*)k, st);
      else spectrum_stage_kernel<float, kSrcReal><<<grid, 256, smem, stream>>>(Kf, (const float*)k, st);
    } else {
      spectrum_stage_kernel<float, kSrcInPlace><<<grid, 256, smem, stream>>>(Kf, nullptr, st);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    pre *= R[j];
  }
  return cudaSuccess;
}

// Standalone real FFTs of length N = R0*R1*R2 over `rows` rows, through the digit stages in the caller's
// workspace W [rows][N] and one gather into natural order.
cudaError_t launch_rfft(const void* x, bool x_bf16, int rows, float2* X, float2* W, const int* R, int S, int sms,
                        cudaStream_t stream) {
  cudaError_t e = launch_spectrum(W, x, x_bf16, kLayoutFull, rows, R, S, stream, false, -1, 0);
  if (e != cudaSuccess) return e;
  fft_gather_kernel<false><<<sms * 8, 256, 0, stream>>>(W, X, rows, R[0], R[1], S > 2 ? R[2] : 1);
  return cudaGetLastError();
}

cudaError_t launch_irfft(const float2* X, int rows, float* x, float2* W, const int* R, int S, int sms,
                         cudaStream_t stream) {
  cudaError_t e = launch_spectrum(W, X, false, 0, rows, R, S, stream, true, -1, 0);
  if (e != cudaSuccess) return e;
  fft_gather_kernel<true><<<sms * 8, 256, 0, stream>>>(W, x, rows, R[0], R[1], S > 2 ? R[2] : 1);
  return cudaGetLastError();
}

}  // namespace sffft
