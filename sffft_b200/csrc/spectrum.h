// Host launchers of the digit-stage kernels (spectrum.cu) and of the block-convolution kernels (blocks.cu).
#pragma once
#include <cuda_runtime.h>

namespace sffft {

// Filter spectrum (or forward DFT) of H rows in digit order for radices R[0..S-1]; see spectrum.cu.
cudaError_t launch_spectrum(float2* Kf, const void* k, bool k_bf16, int layout, int H, const int* R, int S,
                            cudaStream_t stream, bool hermitian, long long kpitch, long long koff);
// Standalone real FFTs of length R[0]*...*R[S-1] over `rows` rows in the workspace W.
cudaError_t launch_rfft(const void* x, bool x_bf16, int rows, float2* X, float2* W, const int* R, int S, int sms,
                        cudaStream_t stream);
cudaError_t launch_irfft(const float2* X, int rows, float* x, float2* W, const int* R, int S, int sms,
                         cudaStream_t stream);

// Block convolution of composite plans; see blocks.cu.
__host__ __device__ long long part_offset(int d, int P, long long blk);
cudaError_t launch_block_gather(const void* u, float* ub, bool bf16, int B, int H, int Lb, int P, int sms,
                                cudaStream_t stream);
cudaError_t launch_block_sum(const float* parts, void* y, bool bf16, int B, int H, int Lb, int P, int sms,
                             cudaStream_t stream);

}  // namespace sffft
