// Registry of compiled fused-kernel instances, one entry per catalog plan.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace sffft {

struct ConvParams;
typedef cudaError_t (*ConvLaunchFn)(const ConvParams& prm, int grid, int smem_bytes, cudaStream_t st);

struct ConvEntry {
  const char* name;            // "64x32/w4"
  int R0, R1, R2, G, W, N, L, threads;
  int bmat_bytes[2];           // per I/O type: the DFT-matrix image (bf16 I/O: no lo set on three-stage plans)
  int smem_bytes[2], tmem_cols[2], slots[2], kslots[2];   // per I/O type (fp32, bf16)
  ConvLaunchFn launch[2][2];   // [io: 0 fp32, 1 bf16][acc: 0 fp32, 1 fp16]
  const void* func[2][2];      // kernel function pointers (attributes, occupancy)
  // small-launch variants with 1 and 2 slots ([0]: 1 slot, [1]: 2 slots; null where not compiled), for launches
  // with at most one or two groups per SM
  ConvLaunchFn launch_small[2][2][2];
  const void* func_small[2][2][2];
  int smem_small[2][2];        // [variant][io]
  void (*build_bmat[2])(uint8_t* img);   // host builders of the cached DFT-matrix images, per I/O type
};

// The two launches of a composite plan's partitioned convolution on block plan `name` (fused_conv_kernel modes
// 1 = forward, 2 = inverse), compiled for the block plans in block_mode_plans (catalog.h).
struct BlockEntry {
  const char* name;
  ConvLaunchFn launch[2][2][2];   // [mode - 1][io][acc]
  const void* func[2][2][2];
  int smem_bytes[2];              // per I/O type
};

// Each translation unit kernels_<part>.cu registers the catalog entries of its size range.
int entries_small(const ConvEntry** out);   // N <= 2048
int entries_mid(const ConvEntry** out);     // N = 4096, 8192
int entries_large(const ConvEntry** out);   // N >= 16384
int block_entries_2stage(const BlockEntry** out);   // composite block plans with two stages
int block_entries_3stage(const BlockEntry** out);   // and with three

}  // namespace sffft
