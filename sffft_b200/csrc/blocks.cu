// Row energies and spectrum sums of composite plans (L = P * Lb above the largest single-pass length; the
// multi-pass plans the reference lists as missing, README.md:175).
//
// A composite plan's partitioned convolution (stages.h, "Partitioned convolution") scales each row by the power
// of two that its energy gives, with one scale for all of a row's blocks, so the energy is taken over the whole
// row here, before the forward launch: E[row] = (Lb / L) * sum_n u[row][n]^2, normalised to Lb values because
// the kernel's scale rule compares the energy with its block length.  One CTA per row, 16-byte loads.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "spectrum.h"

namespace sffft {

__device__ __forceinline__ float sq4(const float* p) {
  const float4 v = __ldg(reinterpret_cast<const float4*>(p));
  return v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
}
__device__ __forceinline__ float sq4(const __nv_bfloat16* p) {
  const uint2 w = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.y));
  return a.x * a.x + a.y * a.y + b.x * b.x + b.y * b.y;
}

template <class T>
__global__ void __launch_bounds__(256) row_energy_kernel(const T* __restrict__ u, float* __restrict__ E, int L,
                                                         float norm) {
  __shared__ float part[8];
  const T* row = u + (size_t)blockIdx.x * L;
  float s = 0.f;
  for (int i = 4 * threadIdx.x; i < L; i += 4 * blockDim.x) s += sq4(row + i);
  for (int m = 16; m > 0; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < 8; w++) t += part[w];
    E[blockIdx.x] = t * norm;
  }
}

cudaError_t launch_row_energy(const void* u, bool bf16, long long rows, int L, int Lb, float* E, cudaStream_t stream) {
  if (rows < 1 || rows > 0x7fffffffLL || L % 4) return cudaErrorInvalidValue;
  const float norm = (float)Lb / (float)L;   // a power of two
  if (bf16)
    row_energy_kernel<__nv_bfloat16><<<(unsigned)rows, 256, 0, stream>>>((const __nv_bfloat16*)u, E, L, norm);
  else
    row_energy_kernel<float><<<(unsigned)rows, 256, 0, stream>>>((const float*)u, E, L, norm);
  return cudaGetLastError();
}

// The spectrum sums of a composite plan's partitioned convolution, in place: for every pair (hb, j) and frequency
// position f, W_p[f] = sum_{q <= p} Z_q[f] K'_{p-q}[f] overwrites Z_p[f] (Z [Hb * P][PB][N], K' [P][Hb][N], complex
// fp32).  One thread per (hb, f) keeps the channel's P filter values K'_d[f] in registers and, for each of the PB
// pairs of the channel, the pair's P values Z_q[f], writing the P sums from the last block down, so each sum reads
// only values not yet overwritten.  Consecutive threads take consecutive f, so every load and store of a warp is one
// contiguous 256-byte run, and each filter value is read from memory once.
template <int NP>
__global__ void __launch_bounds__(256) spectrum_sum_kernel(float2* __restrict__ Z, const float2* __restrict__ K, int Hb,
                                                           int PB, int lgN) {
  const int N = 1 << lgN;
  const long long total = (long long)Hb << lgN;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int hb = (int)(i >> lgN), f = (int)(i & (N - 1));
    float2 k[NP];
#pragma unroll
    for (int d = 0; d < NP; d++) k[d] = __ldg(K + ((long long)d * Hb + hb) * N + f);
    for (int j = 0; j < PB; j++) {
      float2 z[NP];
#pragma unroll
      for (int q = 0; q < NP; q++) z[q] = Z[(((long long)hb * NP + q) * PB + j) * N + f];
#pragma unroll
      for (int p = NP - 1; p >= 0; p--) {
        float re = 0.f, im = 0.f;
#pragma unroll
        for (int q = 0; q <= p; q++) {
          const float2 a = z[q], b = k[p - q];
          re += a.x * b.x - a.y * b.y;
          im += a.x * b.y + a.y * b.x;
        }
        Z[(((long long)hb * NP + p) * PB + j) * N + f] = make_float2(re, im);
      }
    }
  }
}

cudaError_t launch_spectrum_sum(float* Z, const float* K, int Hb, int PB, int N, int P, int sms, cudaStream_t stream) {
  float2* z = reinterpret_cast<float2*>(Z);
  const float2* k = reinterpret_cast<const float2*>(K);
  const unsigned grid = (unsigned)sms * 8;
  int lgN = 0;
  while ((1 << lgN) < N) lgN++;
  switch (P) {
    case 2: spectrum_sum_kernel<2><<<grid, 256, 0, stream>>>(z, k, Hb, PB, lgN); break;
    case 4: spectrum_sum_kernel<4><<<grid, 256, 0, stream>>>(z, k, Hb, PB, lgN); break;
    case 8: spectrum_sum_kernel<8><<<grid, 256, 0, stream>>>(z, k, Hb, PB, lgN); break;
    case 16: spectrum_sum_kernel<16><<<grid, 256, 0, stream>>>(z, k, Hb, PB, lgN); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace sffft
