// Host-side numeric helpers: IEEE float <-> half conversion and the DFT-matrix table builder used
// for the "cached" kernel mode (the same image the kernel builds in "legacy" mode).
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>

#include "stages.h"

namespace sffft {
namespace hostmath {

inline float h2f(uint16_t h) {
  const uint32_t s = (h >> 15) & 1, e = (h >> 10) & 31, m = h & 1023;
  float v;
  if (e == 0) v = std::ldexp((float)m, -24);
  else if (e == 31) v = m ? NAN : INFINITY;
  else v = std::ldexp((float)(m | 1024), (int)e - 25);
  return s ? -v : v;
}

// IEEE round-to-nearest-even float -> half.
inline uint16_t f2h(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0));
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);
  if (ax < 0x38800000u) return (uint16_t)(sign | (uint32_t)std::nearbyint(std::fabs(f) * 16777216.0f));
  const uint32_t e = (ax >> 23) - 112, m = ax & 0x7FFFFFu;
  uint32_t hm = (e << 10) | (m >> 13);
  const uint32_t rem = m & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (hm & 1))) hm++;
  return (uint16_t)(sign | hm);
}

struct BmatEmit {
  uint8_t* img;
  void operator()(int off, int R, int q, int which, int set) {
    const double a = 2.0 * M_PI * (double)q / (double)R;
    const double v = which == 0 ? std::cos(a) : (which == 1 ? -std::sin(a) : std::sin(a));
    uint16_t h = f2h((float)v);
    if (set == 1) h = f2h((float)(v - (double)h2f(h)));
    std::memcpy(img + off, &h, 2);
  }
};

template <class P>
void build_bmat_image(uint8_t* img) {
  BmatEmit e{img};
  for_each_bmat_entry<P>(e, 0, 1);
}

}  // namespace hostmath
}  // namespace sffft
