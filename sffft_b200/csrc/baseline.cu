// cuFFT baseline pipeline on the same device, timed beside the fused kernel.
//
// Same calls as the reference's baseline (sfFFT src/sffft.cu:289-305, 365-371): the filter
// spectrum is a batched C2C forward FFT of the zero-padded filter, halved and scaled by 1/N; each run
// is pad(u) -> R2C -> multiply -> C2R -> slice ("full") or R2C -> multiply -> C2R ("core").
// The small elementwise kernels are this project's own.
#include <cufft.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "status.h"

namespace sffft {

__global__ void bl_half_spectrum(const cufftComplex* Kc, float2* Kh, int H, int N) {
  const int M = N / 2 + 1;
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= (size_t)H * M) return;
  const size_t h = i / M, f = i % M;
  const cufftComplex q = Kc[h * N + f];
  Kh[i] = make_float2(q.x / N, q.y / N);
}
__global__ void bl_pad_filter(const float* k, cufftComplex* kc, int H, int L) {
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= (size_t)H * 2 * L) return;
  const size_t h = i / (2 * L), n = i % (2 * L);
  kc[i] = make_cuComplex(n < (size_t)L ? k[h * L + n] : 0.f, 0.f);
}
__global__ void bl_pad(const float* u, float* up, size_t BH, int L) {
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= BH * 2 * L) return;
  const size_t s = i / (2 * L), n = i % (2 * L);
  up[i] = n < (size_t)L ? u[s * L + n] : 0.f;
}
__global__ void bl_mul(cufftComplex* U, const float2* Kh, size_t BH, int H, int M) {
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= BH * M) return;
  const size_t s = i / M, f = i % M, h = s % H;
  const float2 q = Kh[h * M + f];
  const cufftComplex a = U[i];
  U[i] = make_cuComplex(a.x * q.x - a.y * q.y, a.x * q.y + a.y * q.x);
}
__global__ void bl_slice(const float* yp, float* y, size_t BH, int L) {
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= BH * L) return;
  const size_t s = i / L, n = i % L;
  y[i] = yp[s * 2 * L + n];
}

struct Baseline {
  int L, N, B, H, device;
  cufftHandle pf = 0, pi = 0;
  float* up = nullptr;
  cufftComplex* U = nullptr;
  float* yp = nullptr;
  float2* Kh = nullptr;
};

static unsigned blocks(size_t n) { return (unsigned)((n + 255) / 256); }

int baseline_create(Baseline** out, int L, int B, int H, const float* k_dev, int device) {
  if (!out || !k_dev || L < 1 || B < 1 || H < 1) return SFFFT_ERR_INVALID_ARGUMENT;
  if (cudaSetDevice(device) != cudaSuccess) return SFFFT_ERR_CUDA;
  Baseline* b = new Baseline();
  b->L = L; b->N = 2 * L; b->B = B; b->H = H; b->device = device;
  const size_t BH = (size_t)B * H, M = (size_t)L + 1;
  cufftComplex* Kc = nullptr;
  bool ok = cudaMalloc(&b->up, BH * b->N * sizeof(float)) == cudaSuccess &&
            cudaMalloc(&b->U, BH * M * sizeof(cufftComplex)) == cudaSuccess &&
            cudaMalloc(&b->yp, BH * b->N * sizeof(float)) == cudaSuccess &&
            cudaMalloc(&b->Kh, (size_t)H * M * sizeof(float2)) == cudaSuccess &&
            cudaMalloc(&Kc, (size_t)H * b->N * sizeof(cufftComplex)) == cudaSuccess;
  if (ok) {
    bl_pad_filter<<<blocks((size_t)H * b->N), 256>>>(k_dev, Kc, H, L);
    cufftHandle pk;
    ok = cufftPlan1d(&pk, b->N, CUFFT_C2C, H) == CUFFT_SUCCESS;
    if (ok) {
      ok = cufftExecC2C(pk, Kc, Kc, CUFFT_FORWARD) == CUFFT_SUCCESS;
      cufftDestroy(pk);
    }
    if (ok) bl_half_spectrum<<<blocks((size_t)H * M), 256>>>(Kc, b->Kh, H, b->N);
    ok = ok && cufftPlan1d(&b->pf, b->N, CUFFT_R2C, (int)BH) == CUFFT_SUCCESS &&
         cufftPlan1d(&b->pi, b->N, CUFFT_C2R, (int)BH) == CUFFT_SUCCESS;
    ok = ok && cudaDeviceSynchronize() == cudaSuccess;
  }
  cudaFree(Kc);
  if (!ok) {
    if (b->pf) cufftDestroy(b->pf);
    if (b->pi) cufftDestroy(b->pi);
    cudaFree(b->up); cudaFree(b->U); cudaFree(b->yp); cudaFree(b->Kh);
    delete b;
    return SFFFT_ERR_CUDA;
  }
  *out = b;
  return SFFFT_OK;
}

int baseline_run(Baseline* b, const float* u, float* y, int full, cudaStream_t st) {
  if (!b) return SFFFT_ERR_INVALID_ARGUMENT;
  const size_t BH = (size_t)b->B * b->H, M = (size_t)b->L + 1;
  if (cufftSetStream(b->pf, st) != CUFFT_SUCCESS || cufftSetStream(b->pi, st) != CUFFT_SUCCESS) return SFFFT_ERR_CUDA;
  if (full) bl_pad<<<blocks(BH * b->N), 256, 0, st>>>(u, b->up, BH, b->L);
  if (cufftExecR2C(b->pf, b->up, b->U) != CUFFT_SUCCESS) return SFFFT_ERR_CUDA;
  bl_mul<<<blocks(BH * M), 256, 0, st>>>(b->U, b->Kh, BH, b->H, (int)M);
  if (cufftExecC2R(b->pi, b->U, b->yp) != CUFFT_SUCCESS) return SFFFT_ERR_CUDA;
  if (full) bl_slice<<<blocks(BH * b->L), 256, 0, st>>>(b->yp, y, BH, b->L);
  return cudaGetLastError() == cudaSuccess ? SFFFT_OK : SFFFT_ERR_CUDA;
}

void baseline_destroy(Baseline* b) {
  if (!b) return;
  cudaSetDevice(b->device);
  cufftDestroy(b->pf); cufftDestroy(b->pi);
  cudaFree(b->up); cudaFree(b->U); cudaFree(b->yp); cudaFree(b->Kh);
  delete b;
}

}  // namespace sffft
