// Fused-kernel instances for catalog plans with 16384 <= N <= 65536 (compiled separately for build parallelism).
#include "kernels_impl.cuh"

namespace sffft {
int entries_large(const ConvEntry** out) {
  static const std::vector<ConvEntry> v = collect_entries<16384, 65536>();
  *out = v.data();
  return (int)v.size();
}
}  // namespace sffft
