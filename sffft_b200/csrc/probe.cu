// Layout probe: one tcgen05.mma with the same layout writers and descriptors the fused kernel uses,
// dumping the raw TMEM accumulator.  A GPU test compares it with a host GEMM for each operand layout
// (MN-major 128-B swizzle, K-major 32/64/128-B swizzle with K-slice start offsets) and for the fp16
// accumulator format, so a layout mismatch is attributed to the exact operand form.
#include <cuda_runtime.h>
#include <stdint.h>

#include "plan.h"
#include "status.h"
#include "tc.cuh"

namespace sffft {

// a_kind: 0 MN-major SW128 (64-row blocks, MB = 2), 32/64/128: K-major with that row pitch.
// a_slice: K-slice (16 elements) of the operand row where the tile sits (start address advanced).
struct ProbeArgs {
  const uint16_t* A;   // 128 x 16 row-major
  const uint16_t* Bm;  // n x 16 row-major (B[n][k])
  uint32_t* D;         // 128 x n raw TMEM words
  int a_kind, a_slice, b_pitch, b_slice, n, acc16;
  int* status;
};

__global__ void __launch_bounds__(128, 1) umma_probe_kernel(ProbeArgs pa) {
  __shared__ __align__(1024) uint8_t sm[8 * 4096];   // A region [0, 16K), B region [16K, 32K)
  __shared__ uint64_t bar;
  __shared__ uint32_t slot;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (warp == 0) { tmem_alloc(&slot, 256); tmem_relinquish(); }
  if (tid == 32) { mbar_init(&bar, 1); fence_mbar_init(); }
  for (int i = tid; i < 8 * 4096 / 4; i += 128) reinterpret_cast<uint32_t*>(sm)[i] = 0;
  __syncthreads();
  uint8_t* A = sm;
  uint8_t* Bs = sm + 16384;
  for (int i = tid; i < 128 * 16; i += 128) {
    const int m = i / 16, k = i % 16 + 16 * pa.a_slice;
    const uint32_t off = pa.a_kind == 0 ? mn_off(m, k, 2) : km_off(m, k, pa.a_kind);
    *reinterpret_cast<uint16_t*>(A + off) = pa.A[i];
  }
  for (int i = tid; i < pa.n * 16; i += 128) {
    const int nn = i / 16, k = i % 16 + 16 * pa.b_slice;
    *reinterpret_cast<uint16_t*>(Bs + km_off(nn, k, pa.b_pitch)) = pa.Bm[i];
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = slot;
  if (tid == 0) {
    uint64_t ad;
    if (pa.a_kind == 0) ad = make_sdesc(smem_u32(A) + (uint32_t)(2 * pa.a_slice * 2 * 1024), 1024, 2 * 1024, LT_SW128);
    else ad = make_sdesc(smem_u32(A) + 32u * pa.a_slice, 16, 8 * pa.a_kind, lt_for_pitch(pa.a_kind));
    const uint64_t bd = make_sdesc(smem_u32(Bs) + 32u * pa.b_slice, 16, 8 * pa.b_pitch, lt_for_pitch(pa.b_pitch));
    const uint32_t idesc = make_idesc(128, pa.n, !pa.acc16, pa.a_kind == 0, false);
    mma_f16_ss(tmem, ad, bd, idesc, 0u);
    mma_commit(&bar);
  }
  const bool ok = mbar_wait_bounded(&bar, 0, 1000000000ull);
  if (__syncthreads_and(ok)) {
    tc_fence_after();
    for (int c0 = 0; c0 < pa.n; c0 += 16) {
      uint32_t r[16];
      tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, r);
      tmem_wait_ld();
      for (int j = 0; j < 16; j++) pa.D[(size_t)(warp * 32 + lane) * pa.n + c0 + j] = r[j];
    }
  } else if (tid == 0) {
    atomicExch(pa.status, SFFFT_ERR_TIMEOUT);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// Waits on an mbarrier that nothing arrives at, with a limit of `limit_us` microseconds: exercises the
// bounded-wait path every kernel barrier uses and reports SFFFT_ERR_TIMEOUT through the status word.
__global__ void wait_timeout_kernel(int* status, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) { mbar_init(&bar, 1); fence_mbar_init(); }
  __syncthreads();
  const bool ok = mbar_wait_bounded(&bar, 0, limit_ns);
  if (!__syncthreads_and(ok) && threadIdx.x == 0) atomicExch(status, SFFFT_ERR_TIMEOUT);
}

int wait_timeout_probe(int limit_us) {
  if (limit_us < 1 || limit_us > 1000000) return SFFFT_ERR_INVALID_ARGUMENT;
  int* dS = nullptr;
  int st = 0, rc = SFFFT_ERR_CUDA;
  if (cudaMalloc(&dS, 4) == cudaSuccess && cudaMemset(dS, 0, 4) == cudaSuccess) {
    wait_timeout_kernel<<<1, 64>>>(dS, (unsigned long long)limit_us * 1000ull);
    if (cudaGetLastError() == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess &&
        cudaMemcpy(&st, dS, 4, cudaMemcpyDeviceToHost) == cudaSuccess)
      rc = st;
  }
  cudaFree(dS);
  return rc;
}

int umma_probe(int a_kind, int a_slice, int b_pitch, int b_slice, int n, int acc16, const uint16_t* A_host,
               const uint16_t* B_host, uint32_t* D_host) {
  if (!(a_kind == 0 || a_kind == 32 || a_kind == 64 || a_kind == 128)) return SFFFT_ERR_INVALID_ARGUMENT;
  if (!(b_pitch == 32 || b_pitch == 64 || b_pitch == 128) || n < 16 || n > 128 || n % 16) return SFFFT_ERR_INVALID_ARGUMENT;
  const int a_pitch_slices = a_kind == 0 ? 4 : a_kind / 32;
  if (a_slice < 0 || a_slice >= a_pitch_slices || b_slice < 0 || b_slice >= b_pitch / 32) return SFFFT_ERR_INVALID_ARGUMENT;
  if (a_kind != 0 && 128 * a_kind > 16384) return SFFFT_ERR_INVALID_ARGUMENT;
  uint16_t *dA = nullptr, *dB = nullptr;
  uint32_t* dD = nullptr;
  int* dS = nullptr;
  int rc = SFFFT_ERR_CUDA, st = 0;
  if (cudaMalloc(&dA, 128 * 16 * 2) == cudaSuccess && cudaMalloc(&dB, n * 16 * 2) == cudaSuccess &&
      cudaMalloc(&dD, 128 * n * 4) == cudaSuccess && cudaMalloc(&dS, 4) == cudaSuccess &&
      cudaMemcpy(dA, A_host, 128 * 16 * 2, cudaMemcpyHostToDevice) == cudaSuccess &&
      cudaMemcpy(dB, B_host, n * 16 * 2, cudaMemcpyHostToDevice) == cudaSuccess && cudaMemset(dS, 0, 4) == cudaSuccess) {
    ProbeArgs pa{dA, dB, dD, a_kind, a_slice, b_pitch, b_slice, n, acc16, dS};
    umma_probe_kernel<<<1, 128>>>(pa);
    if (cudaGetLastError() == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess &&
        cudaMemcpy(D_host, dD, 128 * n * 4, cudaMemcpyDeviceToHost) == cudaSuccess &&
        cudaMemcpy(&st, dS, 4, cudaMemcpyDeviceToHost) == cudaSuccess)
      rc = st ? st : SFFFT_OK;
  }
  cudaFree(dA); cudaFree(dB); cudaFree(dD); cudaFree(dS);
  return rc;
}

}  // namespace sffft
