// Row energies of composite plans (L = P * Lb above the largest single-pass length; the multi-pass plans the
// reference lists as missing, README.md:175).
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

}  // namespace sffft
