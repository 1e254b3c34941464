// Instantiates the fused kernel for the catalog entries whose N lies in [NMIN, NMAX].
#pragma once
#include <vector>

#include "catalog.h"
#include "fused_conv.cuh"
#include "hostmath.h"
#include "registry.h"

namespace sffft {

template <class P, class TIO, bool ACC16>
cudaError_t launch_conv(const ConvParams& prm, int grid, int smem_bytes, cudaStream_t st) {
  fused_conv_kernel<P, TIO, ACC16><<<grid, Shape<P, sizeof(TIO)>::NT, smem_bytes, st>>>(prm);
  return cudaGetLastError();
}

template <class P>
ConvEntry make_entry(const char* name) {
  ConvEntry e;
  e.name = name;
  e.R0 = P::R0; e.R1 = P::R1; e.R2 = P::R2; e.G = P::G; e.W = P::W; e.N = P::N; e.L = P::L;
  using S4 = Shape<P, 4>;
  using S2 = Shape<P, 2>;
  e.threads = S4::NT; e.bmat_bytes = P::BMAT_BYTES;
  e.smem_bytes[0] = S4::SMEM; e.smem_bytes[1] = S2::SMEM;
  e.tmem_cols[0] = S4::TMEM_ALLOC; e.tmem_cols[1] = S2::TMEM_ALLOC;
  e.slots[0] = S4::NSLOT; e.slots[1] = S2::NSLOT;
  e.kslots[0] = S4::KSLOT; e.kslots[1] = S2::KSLOT;
  e.launch[0][0] = &launch_conv<P, float, false>;
  e.launch[0][1] = &launch_conv<P, float, true>;
  e.launch[1][0] = &launch_conv<P, __nv_bfloat16, false>;
  e.launch[1][1] = &launch_conv<P, __nv_bfloat16, true>;
  e.func[0][0] = (const void*)&fused_conv_kernel<P, float, false>;
  e.func[0][1] = (const void*)&fused_conv_kernel<P, float, true>;
  e.func[1][0] = (const void*)&fused_conv_kernel<P, __nv_bfloat16, false>;
  e.func[1][1] = (const void*)&fused_conv_kernel<P, __nv_bfloat16, true>;
  e.build_bmat = &hostmath::build_bmat_image<P>;
  return e;
}

template <int NMIN, int NMAX>
std::vector<ConvEntry> collect_entries() {
  std::vector<ConvEntry> v;
#define SF_COLLECT(R0, R1, R2, G, W, NAME)                                              \
  if constexpr (R0 * R1 * R2 >= NMIN && R0 * R1 * R2 <= NMAX) {                        \
    v.push_back(make_entry<Plan<R0, R1, R2, G, W>>(NAME));                              \
  }
  SFFFT_CATALOG(SF_COLLECT)
#undef SF_COLLECT
  return v;
}

}  // namespace sffft
