// Fused-kernel instances for catalog plans with 0 <= N <= 2048 (compiled separately for build parallelism).
#include "kernels_impl.cuh"

namespace sffft {
int entries_small(const ConvEntry** out) {
  static const std::vector<ConvEntry> v = collect_entries<0, 2048>();
  *out = v.data();
  return (int)v.size();
}
}  // namespace sffft
