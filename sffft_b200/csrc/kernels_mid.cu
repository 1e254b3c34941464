// Fused-kernel instances for catalog plans with 4096 <= N <= 8192 (compiled separately for build parallelism).
#include "kernels_impl.cuh"

namespace sffft {
int entries_mid(const ConvEntry** out) {
  static const std::vector<ConvEntry> v = collect_entries<4096, 8192>();
  *out = v.data();
  return (int)v.size();
}
}  // namespace sffft
