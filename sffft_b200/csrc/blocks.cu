// Block convolution for L > 16384 (the multi-pass plans the reference lists as missing, README.md:175):
// a composite plan cuts u and k into P blocks of the block plan's length Lb (L = P * Lb).  With the lag
// d = p - q between output block p and input block q, the output is
//
//   y_p = causal(u_p, k[0 : Lb]) + sum_{d = 1..p} two_sided(u_{p-d}, k[(d-1) Lb + 1 : (d+1) Lb])
//
// (a two-sided filter of 2 Lb - 1 taps covers the lags d Lb - Lb + 1 .. d Lb + Lb - 1 between the two
// blocks).  block_gather_kernel copies u into block-major fp32 [P][B][H][Lb], the host runs the block
// plan's fused kernel with fp32 I/O once per lag d over the P - d input blocks that have a partner (one
// launch of (P - d) * B batch rows), and block_sum_kernel adds the fp32 partial outputs of each output
// block and writes y in the caller's type (bf16 I/O is rounded once, at the end).  Lb and P are powers
// of two.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "spectrum.h"

namespace sffft {

// Element offset of lag d's partial outputs in the parts buffer: sum_{d' < d} (P - d') blocks of B*H*Lb.
__host__ __device__ long long part_offset(int d, int P, long long blk) {
  return blk * ((long long)d * P - (long long)d * (d - 1) / 2);
}

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ld4(const __nv_bfloat16* p) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void st4(__nv_bfloat16* p, float4 v) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  uint2 o;
  o.x = *reinterpret_cast<const uint32_t*>(&a);
  o.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = o;
}

// ub[q][row][t] = u[row][q*Lb + t] in fp32 (row = b*H + h); four consecutive elements per thread.  L and Lb
// are powers of two (lgL, lgLb their logarithms), so the index split is shifts and masks.
template <class T>
__global__ void __launch_bounds__(256) block_gather_kernel(const T* __restrict__ u, float* __restrict__ ub, long long rows,
                                                           int lgL, int lgLb) {
  const long long total4 = rows << (lgL - 2), blk = rows << lgLb;
  const long long cmask = (1ll << lgL) - 1, tmask = (1ll << lgLb) - 1;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total4; i += (long long)gridDim.x * blockDim.x) {
    const long long e = 4 * i, row = e >> lgL, col = e & cmask;
    st4(ub + (col >> lgLb) * blk + (row << lgLb) + (col & tmask), ld4(u + e));
  }
}

// y[row][p*Lb + t] = sum_{d <= p} parts_d[(p - d)*rows + row][t]; four consecutive elements per thread.
template <class T>
__global__ void __launch_bounds__(256) block_sum_kernel(const float* __restrict__ parts, T* __restrict__ y, long long rows,
                                                        int lgL, int lgLb) {
  const int P = 1 << (lgL - lgLb);
  const long long total4 = rows << (lgL - 2), blk = rows << lgLb;
  const long long cmask = (1ll << lgL) - 1, tmask = (1ll << lgLb) - 1;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total4; i += (long long)gridDim.x * blockDim.x) {
    const long long e = 4 * i, row = e >> lgL, col = e & cmask;
    const int p = (int)(col >> lgLb);
    const long long off = (row << lgLb) + (col & tmask);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int d = 0; d <= p; d++) {
      const float4 v = ld4(parts + part_offset(d, P, blk) + (long long)(p - d) * blk + off);
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    st4(y + e, acc);
  }
}

static int log2i(long long v) {
  int r = 0;
  while ((1ll << r) < v) r++;
  return r;
}

cudaError_t launch_block_gather(const void* u, float* ub, bool bf16, int B, int H, int Lb, int P, int sms,
                                cudaStream_t stream) {
  const long long rows = (long long)B * H;
  const int lgLb = log2i(Lb), lgL = lgLb + log2i(P);
  if (bf16)
    block_gather_kernel<__nv_bfloat16><<<sms * 8, 256, 0, stream>>>((const __nv_bfloat16*)u, ub, rows, lgL, lgLb);
  else
    block_gather_kernel<float><<<sms * 8, 256, 0, stream>>>((const float*)u, ub, rows, lgL, lgLb);
  return cudaGetLastError();
}

cudaError_t launch_block_sum(const float* parts, void* y, bool bf16, int B, int H, int Lb, int P, int sms,
                             cudaStream_t stream) {
  const long long rows = (long long)B * H;
  const int lgLb = log2i(Lb), lgL = lgLb + log2i(P);
  if (bf16)
    block_sum_kernel<__nv_bfloat16><<<sms * 8, 256, 0, stream>>>(parts, (__nv_bfloat16*)y, rows, lgL, lgLb);
  else
    block_sum_kernel<float><<<sms * 8, 256, 0, stream>>>(parts, (float*)y, rows, lgL, lgLb);
  return cudaGetLastError();
}

}  // namespace sffft
