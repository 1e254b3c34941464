// Host launchers of the digit-stage kernels (spectrum.cu) and of the composite plans' row energies and spectrum
// sums (blocks.cu).
#pragma once
#include <cuda_runtime.h>

namespace sffft {

// Filter layout of a composite plan's segment d of block length L (launch_spectrum with koff = (d - 1) * L,
// negative for d = 0): kw[n] = k[koff + L + n] = k[d L + n] for n < L and kw[L + m] = k[koff + m] for m < L,
// zero where the index is negative (segment 0 is the causal first block).
constexpr int kLayoutSegment = 4;

// Filter spectrum (or forward DFT) of H rows in digit order for radices R[0..S-1]; see spectrum.cu.
cudaError_t launch_spectrum(float2* Kf, const void* k, bool k_bf16, int layout, int H, const int* R, int S,
                            cudaStream_t stream, bool hermitian, long long kpitch, long long koff);
// Standalone real FFTs of length R[0]*...*R[S-1] over `rows` rows in the workspace W.
cudaError_t launch_rfft(const void* x, bool x_bf16, int rows, float2* X, float2* W, const int* R, int S, int sms,
                        cudaStream_t stream);
cudaError_t launch_irfft(const float2* X, int rows, float* x, float2* W, const int* R, int S, int sms,
                         cudaStream_t stream);

// Row energies of composite plans (sum of squares over each row of L values, times Lb / L); see blocks.cu.
cudaError_t launch_row_energy(const void* u, bool bf16, long long rows, int L, int Lb, float* E, cudaStream_t stream);
// Spectrum sums of composite plans in place: Z_p <- sum_{q <= p} Z_q K'_{p-q} for P = 2, 4, 8 or 16; see blocks.cu.
cudaError_t launch_spectrum_sum(float* Z, const float* K, int Hb, int PB, int N, int P, int sms, cudaStream_t stream);

}  // namespace sffft
