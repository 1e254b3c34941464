// Partitioned-convolution kernels (forward and inverse launches of composite plans) on three-stage block plans
// (compiled separately for build parallelism).
#include "kernels_impl.cuh"

namespace sffft {
int block_entries_3stage(const BlockEntry** out) {
  static const std::vector<BlockEntry> v = collect_block_entries<3>();
  *out = v.data();
  return (int)v.size();
}
}  // namespace sffft
