// Calibration input generator of the sffft CLI: the reference's seeded stream (sfFFT
// src/sffft.cu:308-310) so that calibration batches, and therefore RESULT rows, are comparable with
// the reference program run on the same device: xorshift64 with shifts 13/7/17 from the default state
// 88172645463325252, uniform ((x >> 11) + 0.5) / 2^53, Box-Muller sqrt(-2 ln U1) cos(2 pi U2) with U1
// drawn first.
#pragma once
#include <cmath>
#include <cstddef>

namespace sffft_cli {

struct Rng {
  unsigned long long s = 88172645463325252ULL;
  double uniform() {
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    return ((double)(s >> 11) + 0.5) * (1.0 / 9007199254740992.0);
  }
  double normal() {
    const double u1 = uniform();
    const double u2 = uniform();
    return std::sqrt(-2 * std::log(u1)) * std::cos(2 * M_PI * u2);
  }
};

// Calibration recipe (src/sffft.cu:339-341): u over B*H*L in order, then per-channel decaying filters.
inline void generate(Rng& r, size_t BH, int H, int L, double input_scale, float* u, float* k) {
  for (size_t i = 0; i < BH * (size_t)L; i++) u[i] = (float)(r.normal() * input_scale);
  for (int h = 0; h < H; h++) {
    const double a = 1.0 / (4.0 + (double)L * h / H);
    for (int n = 0; n < L; n++) k[(size_t)h * L + n] = (float)(r.normal() * std::exp(-a * n) * std::sqrt(2 * a));
  }
}

}  // namespace sffft_cli
