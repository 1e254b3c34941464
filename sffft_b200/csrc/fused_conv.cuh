// The fused causal-convolution kernel for sm_100a.
//
// Replaces the reference kernel fftconv<Plan,W,TIO,TAcc,CACHED> (sfFFT src/sffft.cu:243-280).
// One CTA = G pairs of sequences (two batch elements of one channel per pair); the whole working set
// (4*N*G bytes of fp16 data + DFT matrices) stays in shared memory, accumulators live in TMEM.
//
//   setup     warp 0 allocates TMEM; thread 32 initialises the mbarrier; all threads fill the DFT
//             matrices (copy of a cached table, or computed with sincospif: "legacy")
//   input     u (fp32 / bf16) -> fp16 hi+lo, first-stage A operand (MN-major, 128-B swizzle)
//   stages    for sid in 0..2S-1: thread 0 issues the stage's tcgen05.mma's and commits to the
//             mbarrier; every thread waits (bounded), reads its TMEM lane, applies twiddle / spectrum
//             / scale, and writes the next stage's A operand in place (or y for the last stage).
//   teardown  warp 0 frees TMEM.
//
// A barrier wait that exceeds its limit records SFFFT_ERR_TIMEOUT in *status and the CTA skips the
// remaining stages (still freeing TMEM), so a broken pipeline reports an error instead of hanging.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "stages.h"
#include "status.h"
#include "tc.cuh"

namespace sffft {

constexpr unsigned long long kWaitLimitNs = 1000000000ull;   // 1 s per barrier phase

__device__ __forceinline__ float bf16_bits_to_float(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

struct DevOps {
  uint8_t* sm;   // 1024-B aligned base of the data buffer (generic pointer)
  __device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    mma_f16_ss(d, a, b, idesc, acc);
  }
  __device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) { sffft::tmem_ld16(taddr, r); }
  __device__ __forceinline__ void tmem_wait() { tmem_wait_ld(); }
  __device__ __forceinline__ void st16(uint32_t off, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    *reinterpret_cast<uint4*>(sm + off) = make_uint4(a, b, c, d);
  }
  __device__ __forceinline__ void sincospi(float x, float* s, float* c) { sincospif(x, s, c); }
  __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ float lo16f(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu))); }
  __device__ __forceinline__ float hi16f(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }
  template <bool ACC16>
  __device__ __forceinline__ float acc_val_t(uint32_t w) {
    if constexpr (ACC16) return lo16f(w);
    else return __uint_as_float(w);
  }
  bool acc16;
  __device__ __forceinline__ float acc_val(uint32_t w) { return acc16 ? lo16f(w) : __uint_as_float(w); }
  __device__ __forceinline__ void ldK(const float* p, float (&k)[4]) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(p));
    k[0] = v.x; k[1] = v.y; k[2] = v.z; k[3] = v.w;
  }
  __device__ __forceinline__ void load8(const float* p, float* v) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  __device__ __forceinline__ void load8(const __nv_bfloat16* p, float* v) {
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    for (int e = 0; e < 4; e++) { v[2 * e] = bf16_bits_to_float(w[e] & 0xFFFFu); v[2 * e + 1] = bf16_bits_to_float(w[e] >> 16); }
  }
  __device__ __forceinline__ void store1(float* p, float v) { *p = v; }
  __device__ __forceinline__ void store1(__nv_bfloat16* p, float v) { *p = __float2bfloat16(v); }
};

struct BmatEmitDev {
  uint8_t* base;
  __device__ __forceinline__ void operator()(int off, int R, int q, int which, int set) {
    float s, c;
    sincospif(2.0f * (float)q / (float)R, &s, &c);
    const float v = which == 0 ? c : (which == 1 ? -s : s);
    __half h = __float2half_rn(v);
    if (set == 1) {
      // low part of the fp16 hi+lo split (the residual of the fp32 value)
      h = __float2half_rn(v - __half2float(h));
    }
    *reinterpret_cast<__half*>(base + off) = h;
  }
};

struct ConvParams {
  const void* u;
  const float* Kf;       // [H][N] complex fp32 spectrum in digit order (float pairs)
  const uint4* btab;     // cached DFT-matrix image (BMAT_BYTES), or nullptr for in-kernel build
  void* y;
  int* status;
  int B, H;
};

template <class P, class TIO, bool ACC16, int SID>
__device__ __forceinline__ bool run_stages(DevOps& ops, const EpiArgs& ea, uint32_t tmem, uint32_t data_s,
                                           uint32_t bmat_s, uint64_t* bar, int* status) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    tc_fence_after();
    issue_stage<P, ACC16, SID>(ops, tmem, data_s, bmat_s);
    mma_commit(bar);
  }
  bool ok = mbar_wait_bounded(bar, (uint32_t)(SID & 1), kWaitLimitNs);
  ok = __syncthreads_and(ok) != 0;
  if (!ok) {
    if (tid == 0) atomicExch(status, SFFFT_ERR_TIMEOUT);
    return false;
  }
  tc_fence_after();
  {
    constexpr int T = P::tiles(SID);
    const int q = warp & 3;
    for (int t = warp >> 2; t < T; t += P::W / 4) epilogue_row<P, TIO, ACC16, SID>(ops, ea, t, q, lane);
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  if constexpr (SID + 1 < 2 * P::S) return run_stages<P, TIO, ACC16, SID + 1>(ops, ea, tmem, data_s, bmat_s, bar, status);
  return true;
}

template <class P, class TIO, bool ACC16>
__global__ void __launch_bounds__(P::NT, 1) fused_conv_kernel(ConvParams prm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* bmat = sm + P::DATA_BYTES;
  uint64_t* bar = reinterpret_cast<uint64_t*>(bmat + P::BMAT_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5;

  if (warp == 0) { tmem_alloc(tmem_slot, P::TMEM_COLS); tmem_relinquish(); }
  if (tid == 32) { mbar_init(bar, 1); fence_mbar_init(); }

  if (prm.btab) {
    const uint4* src = prm.btab;
    uint4* dst = reinterpret_cast<uint4*>(bmat);
    for (int i = tid; i < P::BMAT_BYTES / 16; i += P::NT) dst[i] = __ldg(src + i);
  } else {
    BmatEmitDev emit{bmat};
    for_each_bmat_entry<P>(emit, tid, P::NT);
  }

  DevOps ops{sm, ACC16};
  load_input<P, TIO>(ops, reinterpret_cast<const TIO*>(prm.u), blockIdx.x, prm.B, prm.H, tid);

  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  EpiArgs ea{tmem, prm.Kf, prm.y, prm.B, prm.H, (int)blockIdx.x};
  run_stages<P, TIO, ACC16, 0>(ops, ea, tmem, smem_u32(sm), smem_u32(bmat), bar, prm.status);

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, P::TMEM_COLS);
}

}  // namespace sffft
