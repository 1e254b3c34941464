// Instantiates the fused kernel for the catalog entries whose N lies in [NMIN, NMAX].
#pragma once
#include <vector>

#include "catalog.h"
#include "fused_conv.cuh"
#include "hostmath.h"
#include "registry.h"

namespace sffft {

// Launched as a programmatic dependent of the stream's previous kernel: the kernel's prologue (barriers, TMEM,
// DFT matrices, twiddle table) may run while that kernel's last CTAs finish; it waits for that kernel to complete
// (griddepcontrol.wait) before it touches anything in global memory the previous work may have produced.
template <class P, class TIO, bool ACC16, int MODE = 0>
cudaError_t launch_conv(const ConvParams& prm, int grid, int smem_bytes, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((unsigned)Shape<P, sizeof(TIO)>::NT);
  cfg.dynamicSmemBytes = (size_t)smem_bytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fused_conv_kernel<P, TIO, ACC16, MODE>, prm);
}

template <class P>
ConvEntry make_entry(const char* name) {
  ConvEntry e;
  e.name = name;
  e.R0 = P::R0; e.R1 = P::R1; e.R2 = P::R2; e.G = P::G; e.W = P::W; e.N = P::N; e.L = P::L;
  using PB = IoPlan<P, 2>;   // the bf16-I/O kernels' plan
  using S4 = Shape<P, 4>;
  using S2 = Shape<PB, 2>;
  e.threads = S4::NT;
  e.bmat_bytes[0] = P::BMAT_BYTES; e.bmat_bytes[1] = PB::BMAT_BYTES;
  e.smem_bytes[0] = S4::SMEM; e.smem_bytes[1] = S2::SMEM;
  e.tmem_cols[0] = S4::TMEM_ALLOC; e.tmem_cols[1] = S2::TMEM_ALLOC;
  e.slots[0] = S4::NSLOT; e.slots[1] = S2::NSLOT;
  e.kslots[0] = S4::KSLOT; e.kslots[1] = S2::KSLOT;
  e.launch[0][0] = &launch_conv<P, float, false>;
  e.launch[0][1] = &launch_conv<P, float, true>;
  e.launch[1][0] = &launch_conv<PB, __nv_bfloat16, false>;
  e.launch[1][1] = &launch_conv<PB, __nv_bfloat16, true>;
  e.func[0][0] = (const void*)&fused_conv_kernel<P, float, false>;
  e.func[0][1] = (const void*)&fused_conv_kernel<P, float, true>;
  e.func[1][0] = (const void*)&fused_conv_kernel<PB, __nv_bfloat16, false>;
  e.func[1][1] = (const void*)&fused_conv_kernel<PB, __nv_bfloat16, true>;
  e.build_bmat[0] = &hostmath::build_bmat_image<P>;
  e.build_bmat[1] = &hostmath::build_bmat_image<PB>;
  for (int v = 0; v < 2; v++)
    for (int io = 0; io < 2; io++) {
      e.smem_small[v][io] = 0;
      for (int a = 0; a < 2; a++) {
        e.launch_small[v][io][a] = nullptr;
        e.func_small[v][io][a] = nullptr;
      }
    }
  return e;
}

// Adds the v-slot variant (v = 1 or 2) of plan P to its entry, where its team splits the conversion evenly (a
// team of 16 warps has more threads than the 8-element runs of the smallest groups).
template <class P, int V>
void add_small_variant(ConvEntry& e) {
  using PV = Plan<P::R0, P::R1, P::R2, P::G, P::W, V>;
  using PVB = IoPlan<PV, 2>;
  constexpr int NT = Shape<PV, 4>::TWARPS * 32, NSQ = 2 * P::G;
  if constexpr (NT % NSQ == 0 && P::L % (8 * (NT / NSQ)) == 0) {
    const int i = V == 1 ? 0 : 1;
    e.smem_small[i][0] = Shape<PV, 4>::SMEM;
    e.smem_small[i][1] = Shape<PVB, 2>::SMEM;
    e.launch_small[i][0][0] = &launch_conv<PV, float, false>;
    e.launch_small[i][0][1] = &launch_conv<PV, float, true>;
    e.launch_small[i][1][0] = &launch_conv<PVB, __nv_bfloat16, false>;
    e.launch_small[i][1][1] = &launch_conv<PVB, __nv_bfloat16, true>;
    e.func_small[i][0][0] = (const void*)&fused_conv_kernel<PV, float, false>;
    e.func_small[i][0][1] = (const void*)&fused_conv_kernel<PV, float, true>;
    e.func_small[i][1][0] = (const void*)&fused_conv_kernel<PVB, __nv_bfloat16, false>;
    e.func_small[i][1][1] = (const void*)&fused_conv_kernel<PVB, __nv_bfloat16, true>;
  }
}

template <class P>
void add_small_variants(ConvEntry& e) {
  add_small_variant<P, 1>(e);
  add_small_variant<P, 2>(e);
}

template <class P>
BlockEntry make_block_entry(const char* name) {
  using PB = IoPlan<P, 2>;
  BlockEntry e;
  e.name = name;
  e.smem_bytes[0] = Shape<P, 4>::SMEM;
  e.smem_bytes[1] = Shape<PB, 2>::SMEM;
  e.launch[0][0][0] = &launch_conv<P, float, false, 1>;
  e.launch[0][0][1] = &launch_conv<P, float, true, 1>;
  e.launch[0][1][0] = &launch_conv<PB, __nv_bfloat16, false, 1>;
  e.launch[0][1][1] = &launch_conv<PB, __nv_bfloat16, true, 1>;
  e.launch[1][0][0] = &launch_conv<P, float, false, 2>;
  e.launch[1][0][1] = &launch_conv<P, float, true, 2>;
  e.launch[1][1][0] = &launch_conv<PB, __nv_bfloat16, false, 2>;
  e.launch[1][1][1] = &launch_conv<PB, __nv_bfloat16, true, 2>;
  e.func[0][0][0] = (const void*)&fused_conv_kernel<P, float, false, 1>;
  e.func[0][0][1] = (const void*)&fused_conv_kernel<P, float, true, 1>;
  e.func[0][1][0] = (const void*)&fused_conv_kernel<PB, __nv_bfloat16, false, 1>;
  e.func[0][1][1] = (const void*)&fused_conv_kernel<PB, __nv_bfloat16, true, 1>;
  e.func[1][0][0] = (const void*)&fused_conv_kernel<P, float, false, 2>;
  e.func[1][0][1] = (const void*)&fused_conv_kernel<P, float, true, 2>;
  e.func[1][1][0] = (const void*)&fused_conv_kernel<PB, __nv_bfloat16, false, 2>;
  e.func[1][1][1] = (const void*)&fused_conv_kernel<PB, __nv_bfloat16, true, 2>;
  return e;
}

template <int STAGES>
std::vector<BlockEntry> collect_block_entries() {
  std::vector<BlockEntry> v;
#define SF_COLLECT_BLK(R0, R1, R2, G, W, NAME)                                                    \
  if constexpr ((R2 > 1 ? 3 : 2) == STAGES && block_mode_plans(R0, R1, R2, W))                   \
    v.push_back(make_block_entry<Plan<R0, R1, R2, G, W>>(NAME));
  SFFFT_CATALOG(SF_COLLECT_BLK)
#undef SF_COLLECT_BLK
  return v;
}

template <int NMIN, int NMAX>
std::vector<ConvEntry> collect_entries() {
  std::vector<ConvEntry> v;
#define SF_COLLECT(R0, R1, R2, G, W, NAME)                                              \
  if constexpr (R0 * R1 * R2 >= NMIN && R0 * R1 * R2 <= NMAX) {                        \
    v.push_back(make_entry<Plan<R0, R1, R2, G, W>>(NAME));                              \
    if constexpr (small_variants(R0, R1, R2, W)) add_small_variants<Plan<R0, R1, R2, G, W>>(v.back()); \
  }
  SFFFT_CATALOG(SF_COLLECT)
#undef SF_COLLECT
  return v;
}

}  // namespace sffft
