// Host emulator of the fused kernel: runs the same stage templates (stages.h) with a CPU backend.
//
// tcgen05.mma is emulated from the raw descriptors: the smem matrix descriptor is decoded (start,
// LBO, SBO, layout type) and operands are read through the canonical UMMA layouts as CUTLASS
// documents them (cute/atom/mma_traits_sm100.hpp, make_umma_desc):
//   K-major, swizzle W (32/64/128 B):  row i -> (i%8)*W + (i/8)*SBO, k -> (k/8)*16 + (k%8)*2
//   MN-major, 128-B swizzle:           m -> (m%64)*2 + (m/64)*LBO,   k -> (k%8)*128 + (k/8)*SBO
// with the swizzle applied to the absolute byte address.  This is deliberately a separate
// transcription from the writers in plan.h, so a mismatch between what an epilogue writes and what a
// descriptor makes the tensor core read shows up here without a GPU.
//
// Exposed through a C entry point for the CPU test-suite; not part of the product path.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "catalog.h"
#include "hostmath.h"
#include "stages.h"

namespace sffft {
namespace emu {

using hostmath::h2f;
using hostmath::f2h;

static inline uint32_t bf16_from_float(float f) {
  uint32_t x; std::memcpy(&x, &f, 4);
  if ((x & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FC0u;
  x += 0x7FFFu + ((x >> 16) & 1u);
  return x >> 16;
}

struct HostOps {
  std::vector<uint8_t>* smem;
  uint32_t base;                 // byte offset of the data buffer that st16 writes
  std::vector<uint32_t>* tmem;   // 128 lanes x 512 columns
  int cur_lane;                  // TMEM lane of the emulated thread
  bool acc16;
  int tmem_cols;                 // columns the kernel allocates
  size_t data_bytes;             // size of the data buffer (epilogue stores must stay inside)

  static uint32_t swz(uint32_t addr, int lt) {
    if (lt == LT_SW128) return addr ^ (((addr >> 7) & 7u) << 4);
    if (lt == LT_SW64) return addr ^ (((addr >> 7) & 3u) << 4);
    if (lt == LT_SW32) return addr ^ (((addr >> 7) & 1u) << 4);
    return addr;
  }
  float rd(uint64_t desc, bool mn, int i, int k) const {
    const uint32_t start = (uint32_t)(desc & 0x3FFFu) << 4, lbo = (uint32_t)((desc >> 16) & 0x3FFFu) << 4,
                   sbo = (uint32_t)((desc >> 32) & 0x3FFFu) << 4;
    const int lt = (int)(desc >> 61);
    uint32_t a;
    if (mn) {
      a = start + (uint32_t)((i % 64) * 2) + (uint32_t)(i / 64) * lbo + (uint32_t)((k % 8) * 128) + (uint32_t)(k / 8) * sbo;
    } else {
      const uint32_t W = lt == LT_SW128 ? 128 : lt == LT_SW64 ? 64 : 32;
      a = start + (uint32_t)(i % 8) * W + (uint32_t)(i / 8) * sbo + (uint32_t)((k / 8) * 16 + (k % 8) * 2);
    }
    a = swz(a, lt);
    if ((size_t)a + 2 > smem->size()) throw std::out_of_range("MMA operand read outside shared memory");
    uint16_t h; std::memcpy(&h, smem->data() + a, 2);
    return h2f(h);
  }
  void mma(uint32_t d, uint64_t ad, uint64_t bd, uint32_t idesc, uint32_t acc) {
    const int N = (int)((idesc >> 17) & 63) * 8, M = (int)((idesc >> 24) & 31) * 16;
    const bool amn = (idesc >> 15) & 1, bmn = (idesc >> 16) & 1, f32 = (idesc >> 4) & 1;
    const int col = (int)(d & 0xFFFF);
    if (col + N > tmem_cols || col < 0) throw std::out_of_range("MMA accumulator outside the TMEM allocation");
    for (int i = 0; i < M; i++)
      for (int n = 0; n < N; n++) {
        double s = 0;
        for (int k = 0; k < 16; k++) s += (double)rd(ad, amn, i, k) * (double)rd(bd, bmn, n, k);
        uint32_t& cell = (*tmem)[(size_t)i * 512 + col + n];
        if (f32) {
          float prev; std::memcpy(&prev, &cell, 4);
          const float v = (float)(s + (acc ? (double)prev : 0.0));
          std::memcpy(&cell, &v, 4);
        } else {
          const float prev = h2f((uint16_t)(cell & 0xFFFF));
          cell = f2h((float)(s + (acc ? (double)prev : 0.0)));
        }
      }
  }
  void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    const int lane = (int)(taddr >> 16) + cur_lane % 32, col = (int)(taddr & 0xFFFF);
    if (lane >= 128 || col + 16 > tmem_cols) throw std::out_of_range("tcgen05.ld outside the TMEM allocation");
    for (int j = 0; j < 16; j++) r[j] = (*tmem)[(size_t)lane * 512 + col + j];
  }
  void tmem_wait() {}
  void st16(uint32_t off, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    const uint32_t w[4] = {a, b, c, d};
    if ((off & 15) || (size_t)off + 16 > data_bytes) throw std::out_of_range("epilogue store outside the data buffer");
    std::memcpy(smem->data() + base + off, w, 16);
  }
  void sincospi(float x, float* s, float* c) {
    *s = (float)std::sin(M_PI * (double)x);
    *c = (float)std::cos(M_PI * (double)x);
  }
  uint32_t pack2(float lo, float hi) { return (uint32_t)f2h(lo) | ((uint32_t)f2h(hi) << 16); }
  float lo16f(uint32_t w) { return h2f((uint16_t)(w & 0xFFFF)); }
  float hi16f(uint32_t w) { return h2f((uint16_t)(w >> 16)); }
  float acc_val(uint32_t w) {
    if (acc16) return h2f((uint16_t)(w & 0xFFFF));
    float f; std::memcpy(&f, &w, 4); return f;
  }
  void ldK(const float* p, float (&k)[4]) { for (int e = 0; e < 4; e++) k[e] = p[e]; }
  void check_z(const float* p) const {
    if (p < z_lo || p + 4 > z_hi) throw std::out_of_range("pair spectrum access outside the workspace");
  }
  void ldZ(const float* p, float (&z)[4]) { check_z(p); for (int e = 0; e < 4; e++) z[e] = p[e]; }
  void stZ(float* p, const float* v) { check_z(p); for (int e = 0; e < 4; e++) p[e] = v[e]; }
  const uint8_t* kst_lo = nullptr;   // staged spectrum region of the current group
  const uint8_t* kst_hi = nullptr;
  void ldsK(const void* p, float (&k)[4]) {
    const uint8_t* b = (const uint8_t*)p;
    if (b < kst_lo || b + 16 > kst_hi) throw std::out_of_range("staged spectrum read outside the staged rows");
    std::memcpy(k, p, 16);
  }
  const uint8_t* in_lo = nullptr;   // the launch's input u (direct global reads must stay inside)
  const uint8_t* in_hi = nullptr;
  void check_in(const void* p, size_t n) const {
    const uint8_t* b = (const uint8_t*)p;
    if (in_lo && (b < in_lo || b + n > in_hi)) throw std::out_of_range("input read outside u");
  }
  void ldraw(const float* p, uint32_t (&w)[8]) { check_in(p, 32); std::memcpy(w, p, 32); }
  void ldraw(const uint16_t* p, uint32_t (&w)[8]) { check_in(p, 16); std::memcpy(w, p, 16); }
  void unpack(const float*, const uint32_t (&w)[8], float* v) { std::memcpy(v, w, 32); }
  void unpack(const uint16_t*, const uint32_t (&w)[8], float* v) {
    for (int e = 0; e < 4; e++) {
      const uint32_t lo = (w[e] & 0xFFFFu) << 16, hi = w[e] & 0xFFFF0000u;
      std::memcpy(&v[2 * e], &lo, 4);
      std::memcpy(&v[2 * e + 1], &hi, 4);
    }
  }
  void store1(float* p, float v) { *p = v; }
  void store1(uint16_t* p, float v) { *p = (uint16_t)bf16_from_float(v); }
  void store4(float* p, const float* v) { for (int i = 0; i < 4; i++) p[i] = v[i]; }
  void store4(uint16_t* p, const float* v) { for (int i = 0; i < 4; i++) p[i] = (uint16_t)bf16_from_float(v[i]); }
  // a sequence's energy (the device sums the SEG lanes that share it with shuffles; the emulated threads run
  // one after another, so they accumulate)
  void energy_store(float* part, int idx, float ss, int) { part[idx] += ss; }
  void st4(uint32_t off, float v) {
    if ((off & 3) || (size_t)off + 4 > data_bytes) throw std::out_of_range("staged output outside the data buffer");
    std::memcpy(smem->data() + base + off, &v, 4);
  }
  void ld4_staged(uint32_t off, uint32_t rot, float* v) {
    if ((off & 15) || (size_t)off + 16 > data_bytes) throw std::out_of_range("staged read outside the data buffer");
    float w[4];
    std::memcpy(w, smem->data() + base + off, 16);
    for (int i = 0; i < 4; i++) v[i] = w[i ^ (int)rot];
  }
  int n_tw;
  const float* z_lo = nullptr;   // composite plans: the pair-spectrum workspace (reads and writes stay inside)
  const float* z_hi = nullptr;
  void tw(int e, float* re, float* im) {
    e &= (n_tw - 1);
    const double a = -2.0 * M_PI * (double)e / (double)n_tw;
    *re = (float)std::cos(a);
    *im = (float)std::sin(a);
  }
  void cmul16(const float* a, const float* b, const float* kk, uint32_t* pr, uint32_t* pim) {
    for (int p = 0; p < 8; p++) {
      float x[2], z[2];
      for (int e = 0; e < 2; e++) {
        const float kr = kk[4 * p + e], ki = kk[4 * p + 2 + e], av = a[2 * p + e], bv = b[2 * p + e];
        x[e] = av * kr - bv * ki;
        z[e] = av * ki + bv * kr;
      }
      pr[p] = pack2(x[0], x[1]);
      pim[p] = pack2(z[0], z[1]);
    }
  }
  // elements j < 8 step from t0, elements j >= 8 from t8 (two recurrences, as on the device)
  void twiddle16(const float* a, const float* b, float t0r, float t0i, float t8r, float t8i, float wr, float wi,
                 uint32_t* pr, uint32_t* pim) {
    float tr = t0r, ti = t0i;
    for (int q = 0; q < 8; q++) {
      if (q == 4) { tr = t8r; ti = t8i; }
      float x[2], z[2];
      for (int e = 0; e < 2; e++) {
        const int j = 2 * q + e;
        x[e] = a[j] * tr - b[j] * ti;
        z[e] = a[j] * ti + b[j] * tr;
        const float nr = tr * wr - ti * wi;
        ti = tr * wi + ti * wr;
        tr = nr;
      }
      pr[q] = pack2(x[0], x[1]);
      pim[q] = pack2(z[0], z[1]);
    }
  }
};

// Stages SID .. of one group: up to 2S - 1, or (MODE 1, a composite plan's forward launch) up to S - 1, whose
// epilogue stores the pair spectra.
template <int SID, int MODE, class P, class TIO, bool ACC16>
void run_stage_emu(HostOps& ops, const EpiArgs& ea, const BlockArgs& ba, const GroupPairs& gp, uint32_t data_s,
                   uint32_t bmat_s) {
  issue_stage<P, ACC16, SID, sizeof(TIO) == 4>(ops, ea.tmem, data_s, bmat_s);
  // every compute warp's share of the stage, in the kernel's unit order (lane quarter q, warp wi of NWQ)
  constexpr int NWQ = Shape<P, (int)sizeof(TIO)>::NWQ;
  for (int wi = 0; wi < NWQ; wi++)
    for (int q = 0; q < 4; q++)
      for (int lane = 0; lane < 32; lane++) {
        ops.cur_lane = lane;
        if constexpr (MODE == 1 && SID == P::S - 1) spec_store_units<P, TIO>(ops, ea, ba, gp, wi, q, lane);
        else epi_warp<P, TIO, ACC16, SID>(ops, ea, gp, wi, q, lane);
      }
  if constexpr (SID == 2 * P::S - 1 && P::S == 3)
    for (int tid = 0; tid < 64; tid++) copy_out_staged<P, TIO>(ops, ea, gp, tid, 64);
  constexpr int LAST = MODE == 1 ? P::S - 1 : 2 * P::S - 1;
  if constexpr (SID < LAST) run_stage_emu<SID + 1, MODE, P, TIO, ACC16>(ops, ea, ba, gp, data_s, bmat_s);
}

// Emulates the persistent kernel's per-group flow: the team's conversion of the group's input (read
// directly from u, with the kernel's thread count and load batching), then the 2S stages, cycling through
// the kernel's data / TMEM slots.
// MODE 1 / 2: a composite plan's forward / inverse launch over the [B][H][Lb] view (H = channels x blocks), with
// the block arguments ba (pair spectra, row energies).
template <class P, class TIO, bool ACC16, int MODE = 0>
int run_plan(const void* u, const float* Kf, void* y, int B, int H, const BlockArgs* ba = nullptr) {
  using SH = Shape<P, (int)sizeof(TIO)>;
  const int PB = (B + 1) / 2;
  const long long pairs = (long long)PB * H;
  const int ngroups = (int)((pairs + P::G - 1) / P::G);
  std::vector<uint8_t> smem(SH::K_OFF, 0);
  std::vector<uint32_t> tmem(128 * 512, 0);
  hostmath::build_bmat_image<P>(smem.data());
  std::vector<uint8_t> kst;
  const TIO* uu = (const TIO*)u;
  for (int group = 0; group < ngroups; group++) {
    const int slot = group % SH::NSLOT;
    const uint32_t dbase = (uint32_t)(SH::DATA_OFF + slot * P::DATA_BYTES);
    HostOps ops{&smem, dbase, &tmem, 0, ACC16, SH::TMEM_ALLOC, (size_t)P::DATA_BYTES, nullptr, nullptr, nullptr, nullptr, P::N};
    if (u) {
      ops.in_lo = (const uint8_t*)u;
      ops.in_hi = (const uint8_t*)u + (size_t)B * H * P::L * sizeof(TIO);
    }
    const BlockArgs bz = ba ? *ba : BlockArgs{nullptr, nullptr, 0, 0};
    if (ba) {
      ops.z_lo = ba->Z;
      ops.z_hi = ba->Z + 2 * (size_t)((B + 1) / 2) * H * P::N;
    }
    const GroupPairs gp = group_pairs(group, P::G, B, H);
    std::memset(smem.data() + dbase, 0xFF, P::DATA_BYTES);   // poison: stale data must never be read
    constexpr int NT = SH::TWARPS * 32;
    std::vector<float> part(Energy<P, NT>::SLOTS, 0.f);
    EpiArgs ea{(uint32_t)(slot * P::TMEM_COLS), Kf, y, B, H, group, nullptr, 0, part.data()};
    if constexpr (MODE == 0) {
      // the two conversion passes of the kernel: energies, then (where a row needs it) scaled input
      for (int tid = 0; tid < NT; tid++) convert_group<P, TIO, SH::NB, NT>(ops, uu, gp, tid, part.data(), 1.f);
      if (group_rescaled<P, NT>(part.data()))
        for (int tid = 0; tid < NT; tid++) {
          const int j = tid / Energy<P, NT>::TPS;
          convert_group<P, TIO, SH::NB, NT>(ops, uu, gp, tid, nullptr, row_in_scale<P, NT>(part.data(), j >> 1, j & 1));
        }
    } else {
      fill_energies<P, NT>(part.data(), bz, gp, 0, 1);
      if constexpr (MODE == 1) {
        for (int tid = 0; tid < NT; tid++) {
          const int j = tid / Energy<P, NT>::TPS;
          convert_group<P, TIO, SH::NB, NT>(ops, uu, gp, tid, nullptr, row_in_scale<P, NT>(part.data(), j >> 1, j & 1));
        }
        run_stage_emu<0, 1, P, TIO, ACC16>(ops, ea, bz, gp, dbase, 0u);
      } else {
        constexpr int NWQ = SH::NWQ;
        for (int wi = 0; wi < NWQ; wi++)
          for (int q = 0; q < 4; q++)
            for (int lane = 0; lane < 32; lane++) spec_load_units<P, TIO>(ops, bz, gp, wi, q, lane);
        run_stage_emu<P::S, 2, P, TIO, ACC16>(ops, ea, bz, gp, dbase, 0u);
      }
      continue;
    }
    // the loader warp's staging of the group's spectrum rows (same swizzle as the device)
    if constexpr (SH::KSLOT > 0) {
      const int hf = gp.get(0, P::L).h;
      int hl = hf;
      for (int g = P::G - 1; g > 0; g--) {
        const int h = gp.get(g, P::L).h;
        if (h >= 0) { hl = h; break; }
      }
      if (hf >= 0 && hl - hf + 1 <= SH::KC) {
        kst.assign((size_t)SH::KC * SH::KROW, 0xEE);
        constexpr int PPR = P::RL / 2;
        for (int ci = 0; ci <= hl - hf; ci++)
          for (int o = 0; o < SH::KROW / 16; o++) {
            const int rr = o / PPR, rem = o - rr * PPR;
            float pc[4];
            spec_piece(Kf + 2ll * (hf + ci) * P::N + 4 * o, stage_scale(P::RL), pc);
            std::memcpy(kst.data() + (size_t)ci * SH::KROW + kstage_off<P::N, P::RL>(rr, rem >> 3, rem & 7), pc, 16);
          }
        ea.kst = kst.data();
        ea.khf = hf;
        ops.kst_lo = kst.data();
        ops.kst_hi = kst.data() + (size_t)(hl - hf + 1) * SH::KROW;
      }
    }
    run_stage_emu<0, 0, P, TIO, ACC16>(ops, ea, bz, gp, dbase, 0u);
  }
  return 0;
}

// A composite plan "<P>x[<block plan Pl>]": the row energies of the partitioned convolution (fp32 sums over the
// whole row, times Lb / L), then the forward and the inverse launch over the [B][H * P][Lb] view.
template <class Pl, class TIO, bool ACC16>
int run_composite(int P, const void* u, const float* Kf, void* y, int B, int H) {
  const int L = P * Pl::L;
  std::vector<float> En((size_t)B * H);
  for (size_t r = 0; r < En.size(); r++) {
    float s = 0.f;
    for (int n = 0; n < L; n++) {
      float v;
      if constexpr (sizeof(TIO) == 4) v = ((const float*)u)[r * L + n];
      else {
        const uint32_t w = (uint32_t)((const uint16_t*)u)[r * L + n] << 16;
        std::memcpy(&v, &w, 4);
      }
      s += v * v;
    }
    En[r] = s * ((float)Pl::L / (float)L);
  }
  std::vector<float> Z(2 * (size_t)((B + 1) / 2) * H * P * Pl::N, 0.f);
  BlockArgs ba;
  ba.Z = Z.data();
  ba.En = En.data();
  ba.lgP = 0;
  while ((1 << ba.lgP) < P) ba.lgP++;
  ba.Hb = H;
  run_plan<Pl, TIO, ACC16, 1>(u, nullptr, nullptr, B, H * P, &ba);
  // the spectrum sums, in place (the device's spectrum_sum_kernel): Z_p <- sum_{q <= p} Z_q K'_{p-q}, fp32
  const int PB = (B + 1) / 2, N = Pl::N;
  std::vector<float> zq(2 * (size_t)P);
  for (int hb = 0; hb < H; hb++)
    for (int j = 0; j < PB; j++)
      for (int f = 0; f < N; f++) {
        auto zi = [&](int q) { return 2 * ((((size_t)hb * P + q) * PB + j) * N + f); };
        for (int q = 0; q < P; q++) { zq[2 * q] = Z[zi(q)]; zq[2 * q + 1] = Z[zi(q) + 1]; }
        for (int p = P - 1; p >= 0; p--) {
          float re = 0.f, im = 0.f;
          for (int q = 0; q <= p; q++) {
            const float* kk = Kf + 2 * (((size_t)(p - q) * H + hb) * N + f);
            re += zq[2 * q] * kk[0] - zq[2 * q + 1] * kk[1];
            im += zq[2 * q] * kk[1] + zq[2 * q + 1] * kk[0];
          }
          Z[zi(p)] = re;
          Z[zi(p) + 1] = im;
        }
      }
  run_plan<Pl, TIO, ACC16, 2>(nullptr, Kf, y, B, H * P, &ba);
  return 0;
}

// A small-launch variant (fewer, wider teams) where its team splits the conversion evenly, else 2 (unknown).
template <class Pl>
int run_variant(int io, int acc, const void* u, const float* Kf, void* y, int B, int H) {
  constexpr int NT = Shape<Pl, 4>::TWARPS * 32, NSQ = 2 * Pl::G;
  if constexpr (NT % NSQ == 0 && Pl::L % (8 * (NT / NSQ)) == 0) {
    if (io == 0 && acc == 0) return run_plan<Pl, float, false>(u, Kf, y, B, H);
    if (io == 0 && acc == 1) return run_plan<Pl, float, true>(u, Kf, y, B, H);
    if (io == 1 && acc == 0) return run_plan<IoPlan<Pl, 2>, uint16_t, false>(u, Kf, y, B, H);
    return run_plan<IoPlan<Pl, 2>, uint16_t, true>(u, Kf, y, B, H);
  } else {
    return 2;
  }
}

}  // namespace emu
}  // namespace sffft

extern "C" {
// Emulated partitioned convolution of the composite plan "<P>x[<config>]" (config: a block plan with the
// partitioned-convolution kernels); Kf holds the P filter-segment spectra [P][H][N].  Returns as sffft_emu_conv.
int sffft_emu_conv_composite(const char* config, int P, int io, int acc, const void* u, const float* Kf, void* y, int B,
                             int H) {
  using namespace sffft;
  int rc = 2;
  if (P < 2 || (P & (P - 1))) return 2;
  try {
#define SF_EMU_COMPOSITE(R0, R1, R2, G, W, NAME)                                                        \
  if constexpr (block_mode_plans(R0, R1, R2, W)) {                                                     \
    if (std::string(config) == NAME) {                                                                  \
      using Pl = Plan<R0, R1, R2, G, W>;                                                                \
      if (io == 0 && acc == 0) rc = emu::run_composite<Pl, float, false>(P, u, Kf, y, B, H);            \
      else if (io == 0 && acc == 1) rc = emu::run_composite<Pl, float, true>(P, u, Kf, y, B, H);        \
      else if (io == 1 && acc == 0) rc = emu::run_composite<IoPlan<Pl, 2>, uint16_t, false>(P, u, Kf, y, B, H);    \
      else rc = emu::run_composite<IoPlan<Pl, 2>, uint16_t, true>(P, u, Kf, y, B, H);                              \
    }                                                                                                   \
  }
  SFFFT_CATALOG(SF_EMU_COMPOSITE)
#undef SF_EMU_COMPOSITE
  } catch (const std::exception&) {
    return 3;
  }
  return rc;
}

// Runs the emulated fused kernel for catalog entry `config` ("64x32/w4" ...).  io: 0 fp32, 1 bf16 (u,y as
// uint16 bf16 bits).  acc: 0 fp32, 1 fp16.  Returns 0 on success, nonzero for an unknown config.
int sffft_emu_conv(const char* config, int io, int acc, const void* u, const float* Kf, void* y, int B, int H) {
  using namespace sffft;
  int rc = 2;
  try {
#define SF_EMU_CASE(R0, R1, R2, G, W, NAME)                                                           \
  if (std::string(config) == NAME) {                                                                  \
    using Pl = Plan<R0, R1, R2, G, W>;                                                                \
    if (io == 0 && acc == 0) rc = emu::run_plan<Pl, float, false>(u, Kf, y, B, H);                    \
    else if (io == 0 && acc == 1) rc = emu::run_plan<Pl, float, true>(u, Kf, y, B, H);                \
    else if (io == 1 && acc == 0) rc = emu::run_plan<IoPlan<Pl, 2>, uint16_t, false>(u, Kf, y, B, H);            \
    else rc = emu::run_plan<IoPlan<Pl, 2>, uint16_t, true>(u, Kf, y, B, H);                                      \
  }
  SFFFT_CATALOG(SF_EMU_CASE)
#undef SF_EMU_CASE
  // the small-launch variants of the default plans (1 or 2 slots, wider teams): "<name>@1", "<name>@2"
#define SF_EMU_SMALL(R0, R1, R2, G, W, NAME)                                                                \
  for (int v = 1; v <= 2; v++) {                                                                             \
    if (std::string(config) != std::string(NAME) + "@" + std::to_string(v)) continue;                       \
    if (v == 1) rc = emu::run_variant<Plan<R0, R1, R2, G, W, 1>>(io, acc, u, Kf, y, B, H);                  \
    else rc = emu::run_variant<Plan<R0, R1, R2, G, W, 2>>(io, acc, u, Kf, y, B, H);                         \
  }
  SF_EMU_SMALL(16, 16, 1, 8, 8, "16x16/w8") SF_EMU_SMALL(32, 16, 1, 8, 8, "32x16/w8")
  SF_EMU_SMALL(32, 32, 1, 4, 8, "32x32/w8") SF_EMU_SMALL(64, 32, 1, 4, 8, "64x32/w8")
  SF_EMU_SMALL(64, 64, 1, 2, 8, "64x64/w8") SF_EMU_SMALL(32, 16, 16, 1, 8, "32x16x16/w8")
  SF_EMU_SMALL(32, 32, 16, 1, 8, "32x32x16/w8")
#undef SF_EMU_SMALL
  } catch (const std::exception&) {
    return 3;
  }
  return rc;
}
}
