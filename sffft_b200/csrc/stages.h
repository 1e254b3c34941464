// Stage logic of the fused convolution, written once for the device (tcgen05 PTX, fused_conv.cuh)
// and for the host emulator (emu.cpp) through an `Ops` backend:
//   ops.mma(d_tmem, a_desc, b_desc, idesc, accumulate)      tcgen05.mma.cta_group::1.kind::f16
//   ops.tmem_ld16(taddr, r[16]) / ops.tmem_wait()            tcgen05.ld.32x32b.x16 of this lane
//   ops.st16(byte_off, w0..w3)                               16-byte shared-memory store
//   ops.sincospi(x, &s, &c)                                  sin/cos of pi*x
//   ops.pack2(lo, hi)                                        two floats -> f16x2 (round to nearest)
//   ops.acc_val(raw)                                         TMEM word -> float (fp32 or fp16 accumulator)
//   ops.ldK(p) / ops.ldsK(p)                                 four floats (two complex) of the spectrum from
//                                                            global / staged shared memory
//   ops.cmul16(a, b, kk, pr, pim)                            16 complex values x spectrum pieces -> fp16 pairs
//   ops.ldraw(p, w) / ops.unpack(p, w, v)                    eight input values (TIO) from global, as raw words
//                                                            -> float (unpacked when converted)
//   ops.store1(p, v) / ops.store4(p, v[4])                   output values (TIO) to global memory
//   ops.tw(e, &re, &im)                                      w_N^e from the CTA's twiddle table
//   ops.twiddle16(a, b, t0, t8, w, pr, pim)                  16 complex values x t0*w^j (j < 8) and
//                                                            t8*w^(j-8) (j >= 8) -> fp16 pairs
//   ops.st4(off, v) / ops.ld4_staged(off, rot, v)            staged fp32 outputs (3-stage plans)
//
// Algorithm per pair (reference: sfFFT src/sffft.cu:137-280, restated for tcgen05 and pairing):
//   forward digits 0..S-1, each: DFT_R along the digit, x 1/sqrt(R), then the four-step twiddle
//   (src/sffft.cu:106-113) or, after the last digit, the filter spectrum Kf (src/sffft.cu:229-236);
//   inverse digits S-1..0 with conjugate DFTs and conjugate twiddles; the last inverse digit keeps
//   only time rows n0 < R0/2, i.e. outputs n < L (src/sffft.cu:180-181).
#pragma once
#include "plan.h"

namespace sffft {

// Pair bookkeeping for one CTA: pair gp = cta*G + g covers batch elements 2j, 2j+1 of channel h.
struct PairInfo {
  long long off0, off1;   // element offsets of the two sequences in u / y, or -1 when absent
  int h;                  // channel (spectrum row), -1 when the pair slot is empty
  int j;                  // batch pair: rows 2j, 2j + 1
};

// Pair bookkeeping of one group with 32-bit arithmetic: one division per group, then pair g is found
// from the group's first pair: j0 < PB and g < G, so one subtraction suffices whenever PB >= G (batches
// of at least 2G); a division is left only for smaller batches.  2j*H + h < B*H <= INT_MAX.
struct GroupPairs {
  int h0, j0, PB, B, H;
  SF_HD PairInfo get(int g, int L) const {
    int j = j0 + g, h = h0;
    if (j >= PB) {
      j -= PB;
      h++;
      if (j >= PB) { const int d = j / PB; j -= d * PB; h += d; }
    }
    PairInfo pi;
    pi.j = j;
    if (h >= H) { pi.off0 = pi.off1 = -1; pi.h = -1; return pi; }
    pi.h = h;
    pi.off0 = (long long)(2 * j * H + h) * L;
    pi.off1 = (2 * j + 1 < B) ? pi.off0 + (long long)H * L : -1;
    return pi;
  }
};
SF_HD GroupPairs group_pairs(int group, int G, int B, int H) {
  GroupPairs gp;
  gp.PB = (B + 1) / 2; gp.B = B; gp.H = H;
  const int first = group * G;
  gp.h0 = first / gp.PB;
  gp.j0 = first - gp.h0 * gp.PB;
  return gp;
}

SF_HD PairInfo pair_info(int cta, int g, int G, int B, int H, int L) {
  const int PB = (B + 1) / 2;
  const long long gp = (long long)cta * G + g;
  PairInfo pi;
  pi.j = 0;
  if (gp >= (long long)PB * H) { pi.off0 = pi.off1 = -1; pi.h = -1; return pi; }
  const int h = (int)(gp / PB), j = (int)(gp % PB);
  pi.h = h;
  pi.j = j;
  pi.off0 = ((long long)(2 * j) * H + h) * L;
  pi.off1 = (2 * j + 1 < B) ? ((long long)(2 * j + 1) * H + h) * L : -1;
  return pi;
}

// ---------------------------------------------------------------------------------------------
// Input conversion: raw u (two real sequences per pair) -> first-stage A operand, fp16 hi + lo split.
//   element (row m = g*V0 + v, K-row plane*R0 + n0 [hi] / plane*R0 + R0/2 + n0 [lo]), n = n0*V0 + v.
// A group's input is its 2G sequences (sequence j = 2*g + plane, element n), read straight from global
// memory: thread tid of nthreads takes 8 consecutive elements per step and keeps NB steps' loads in flight,
// refilling each register slot with the load NB steps ahead as soon as it has converted the slot (issuing
// NB loads, converting all NB and only then issuing the next NB drained the loads at every batch: 8 %
// slower at L = 1024).  Absent sequences (odd B, past the last pair) read as zero.
// bf16 input within the fp16 range is exact in fp16 (apart from fp16-subnormal values below 6e-5, whose
// residue under 3e-8 is dropped), so it has no lo plane to compute.  Values beyond the fp16 range
// (|x| > 65504, possible in fp32 and bf16 input) become infinite in the hi plane and give inf / NaN
// outputs, as the reference's fp16 conversion does.
//
// A group's 2G sequences are split evenly over the team's NT threads: TPS = NT / 2G consecutive threads per
// sequence, each taking 8 consecutive elements per step, so the steps of a thread stay inside one sequence
// (a warp's step reads 256 consecutive elements, or 32 / TPS whole runs of 8 * TPS) and each thread sums its
// sequence's energy in a register.  A group is converted in one or two passes (see pair_scales below):
//   part != null  first pass: unscaled conversion that also records the energy (sum of squares) of every
//                 sequence, one slot per warp of the sequence (Energy::SPS slots each)
//   part == null  second pass (only for a group with a row to rescale): every value is multiplied by the
//                 power of two `scale` of the thread's sequence before the fp16 split.
// ---------------------------------------------------------------------------------------------
template <class P, int NT>
struct Energy {
  static constexpr int NSQ = 2 * P::G;              // sequences of a group
  static constexpr int TPS = NT / NSQ;              // threads per sequence
  static constexpr int SEG = TPS < 32 ? TPS : 32;   // lanes of a warp that share a sequence
  static constexpr int SPS = TPS / SEG;             // energy slots per sequence (one per warp of it)
  static constexpr int SLOTS = NSQ * SPS;
  static constexpr int NSTEP = P::L / (8 * TPS);    // conversion steps of a thread
  static_assert(NT % NSQ == 0 && P::L % (8 * TPS) == 0, "conversion split");
};

template <class P, class TIO, int NB, int NT, class Ops>
SF_HD void convert_group(Ops& ops, const TIO* u, const GroupPairs& gp, int tid, float* part, float scale) {
  using EN = Energy<P, NT>;
  constexpr int V0 = P::N / P::R0, MB0 = P::MB(0), TPS = EN::TPS, NSTEP = EN::NSTEP;
  const int j = tid / TPS, tl = tid - j * TPS, g = j >> 1, plane = j & 1;   // this thread's sequence
  const PairInfo pi = gp.get(g, P::L);
  const long long soff = plane == 0 ? pi.off0 : pi.off1;
  uint32_t w[NB][8];
  int nb[NB];
  // step i: elements n = tl * 8 + i * 8 * TPS .. + 7 of the sequence
  auto issue = [&](int b, int i) {
    const int n = tl * 8 + i * 8 * TPS;
    nb[b] = n;
    if (soff >= 0) ops.ldraw(u + soff + n, w[b]);
    else {
      for (int q = 0; q < 8; q++) w[b][q] = 0u;   // zero bits read as 0.0 in both formats
    }
  };
  float e2 = 0.f;
  auto finish = [&](int b) {
    float v[8];
    ops.unpack(u, w[b], v);
    if (part) {
      for (int q = 0; q < 8; q++) e2 += v[q] * v[q];
    } else {
      for (int q = 0; q < 8; q++) v[q] *= scale;
    }
    const int n0 = nb[b] / V0, vv = nb[b] - n0 * V0;
    uint32_t hi[4], lo[4];
    for (int q = 0; q < 4; q++) hi[q] = ops.pack2(v[2 * q], v[2 * q + 1]);
    // K-row k + R0/2 (the lo plane) is R0/16 K-groups further: same swizzle phase, since R0/2 % 8 == 0
    const uint32_t off = mn_off(g * V0 + vv, plane * P::R0 + n0, MB0), off_lo = off + (uint32_t)(P::R0 / 16) * MB0 * 1024u;
    ops.st16(off, hi[0], hi[1], hi[2], hi[3]);
    if constexpr (sizeof(TIO) == 4) {
      for (int q = 0; q < 4; q++)
        lo[q] = ops.pack2(v[2 * q] - ops.lo16f(hi[q]), v[2 * q + 1] - ops.hi16f(hi[q]));
      ops.st16(off_lo, lo[0], lo[1], lo[2], lo[3]);
    } else if constexpr (P::R0 == 16) {
      ops.st16(off_lo, 0u, 0u, 0u, 0u);   // bf16 converts exactly: its lo plane is zero
    }
  };
  // A rolled loop: the kernel's code must stay small (its instruction cache is a limit), so the steps are not
  // unrolled beyond the NB loads kept in flight.
#pragma unroll
  for (int b = 0; b < NB; b++)
    if (b < NSTEP) issue(b, b);
#pragma unroll 1
  for (int i0 = 0; i0 < NSTEP; i0 += NB) {
#pragma unroll
    for (int b = 0; b < NB; b++) {
      if (i0 + b >= NSTEP) break;
      finish(b);
      if (i0 + b + NB < NSTEP) issue(b, i0 + b + NB);
    }
  }
  // the sequence's energy over the SEG lanes of this warp that share it, one slot per warp of the sequence
  if (part) ops.energy_store(part, j * EN::SPS + tl / EN::SEG, e2, EN::SEG);
}

// ---------------------------------------------------------------------------------------------
// Per-sequence scaling of pairs.
//
// A pair packs two batch rows into one complex transform, so the fp16 rounding noise of each stage is set by
// the pair's combined magnitude and lands in both rows' outputs.  A row much smaller than its partner would
// then carry the partner's noise: relative error ~ 3.5e-4 * sqrt((1 + E_big / E_small) / 2) for energies
// E = sum u^2 (the reference transforms every row alone, sfFFT src/sffft.cu:249, and has no such coupling).
// The conversion's first pass measures both energies; where they differ by 2x or more, or where the pair's
// rows are all tiny (rms below 2^-6, where fp16 storage would lose digits), the group is converted again
// with each row multiplied by a power of two: the smaller row is brought within a factor sqrt(2) of its
// partner's rms (never above the larger row's level, so the fp16 range -- and the reference's overflow at
// large input scales -- is unchanged for balanced pairs), and tiny pairs are brought up to rms ~1.  The
// output epilogue multiplies each row by the inverse power of two (exact), or by 0 for an all-zero row,
// whose output would otherwise be its partner's rounding noise (and whose exact result is 0).
// Non-finite energies leave the pair unscaled (inf / NaN then propagate as in the reference).  A row whose
// sum of squares underflows fp32 (|u| below ~1e-19) counts as all-zero; the reference's fp16 storage
// flushes such values to zero as well.
// ---------------------------------------------------------------------------------------------
SF_HD float exp2i(int f) {   // 2^f exactly, |f| <= 126
  union {
    uint32_t u;
    float x;
  } c;
  c.u = (uint32_t)(f + 127) << 23;
  return c.x;
}

SF_HD int round_half_log2(float r) {   // round(log2(r) / 2), |result| <= 100
  float f = 0.5f * log2f(r);
  f = f > 100.f ? 100.f : (f < -100.f ? -100.f : f);
  return (int)(f < 0.f ? f - 0.5f : f + 0.5f);
}

// Exponents f0, f1 of the powers of two that scale a pair's two rows, from their energies E0, E1 (sums of
// squares over L values each).
SF_HD void pair_exponents(float E0, float E1, int L, int* f0, int* f1) {
  int f[2] = {0, 0};
  if (E0 <= 3.0e38f && E1 <= 3.0e38f) {   // false for inf and NaN: such pairs stay unscaled
    const float Eb = E0 > E1 ? E0 : E1;
    if (Eb > 0.f && Eb < (float)L * (1.f / 4096.f)) f[0] = f[1] = round_half_log2((float)L / Eb);
    if (E0 > 0.f && E1 > 0.f) {
      const float r = E0 / E1;
      if (r >= 2.f) f[1] += round_half_log2(r);
      else if (r <= 0.5f) f[0] += round_half_log2(1.f / r);
    }
  }
  *f0 = f[0] > 120 ? 120 : f[0];
  *f1 = f[1] > 120 ? 120 : f[1];
}

// Energies of pair g's two rows from the group's energy slots.
template <class P, int NT>
SF_HD void pair_energies(const float* en, int g, float* E0, float* E1) {
  using EN = Energy<P, NT>;
  float e[2] = {0.f, 0.f};
  for (int p = 0; p < 2; p++)
    for (int i = 0; i < EN::SPS; i++) e[p] += en[(2 * g + p) * EN::SPS + i];
  *E0 = e[0];
  *E1 = e[1];
}

// Input scale of row p (0, 1) of pair g.
template <class P, int NT>
SF_HD float row_in_scale(const float* en, int g, int p) {
  float E0, E1;
  int f0, f1;
  pair_energies<P, NT>(en, g, &E0, &E1);
  pair_exponents(E0, E1, P::L, &f0, &f1);
  return exp2i(p ? f1 : f0);
}

// Output scales of pair g's rows: the inverse powers of two, or 0 for an all-zero row.
template <class P, int NT>
SF_HD void pair_out_scales(const float* en, int g, float* o0, float* o1) {
  float E0, E1;
  int f0, f1;
  pair_energies<P, NT>(en, g, &E0, &E1);
  pair_exponents(E0, E1, P::L, &f0, &f1);
  *o0 = E0 == 0.f ? 0.f : exp2i(-f0);
  *o1 = E1 == 0.f ? 0.f : exp2i(-f1);
}

// Whether any row of the group is scaled (the kernel asks this per warp, lanes in parallel).
template <class P, int NT>
SF_HD bool group_rescaled(const float* en) {
  bool any = false;
  for (int g = 0; g < P::G; g++) {
    float E0, E1;
    int f0, f1;
    pair_energies<P, NT>(en, g, &E0, &E1);
    pair_exponents(E0, E1, P::L, &f0, &f1);
    any = any || f0 != 0 || f1 != 0;
  }
  return any;
}

// ---------------------------------------------------------------------------------------------
// MMA issue for stage SID (one thread)
// ---------------------------------------------------------------------------------------------
// Descriptor with its start-address field advanced by `bytes` (shared-memory addresses stay below 2^18,
// so the 14-bit field never carries into the next one).
SF_HD uint64_t sdesc_add(uint64_t desc, uint32_t bytes) { return desc + (uint64_t)(bytes >> 4); }

// LO: the first stage's K axis carries the input's fp16 lo plane (fp32 input).  bf16 input converts to fp16
// exactly, its lo plane is zero, and with R0 >= 32 its K-slices (rows n0 >= R0/2 of each plane) are skipped;
// with R0 == 16 one slice holds both halves and the conversion writes zeros there.
template <class P, bool ACC16, int SID, bool LO, class Ops>
SF_HD void issue_stage(Ops& ops, uint32_t tmem, uint32_t data_s, uint32_t bmat_s) {
  constexpr int R = P::rad(SID), T = P::tiles(SID), NSL = R / 16;
  constexpr bool KM = P::kmajor(SID), INV = P::inv(SID);
  constexpr bool B0 = (SID == 0 && P::R0 == 16);
  constexpr int HS = P::R0 >= 32 ? P::R0 / 32 : 1;           // B K-slices per first-stage half
  constexpr int NJ = (SID == 0 && !B0 && !LO) ? HS : NSL;     // K-slices issued per plane
  constexpr uint32_t idesc = make_idesc(128, 2 * R, !ACC16, !KM, false);
  constexpr int RB = kmaj_data_pitch(R), MBs = P::MB(SID);
  const uint64_t a_base = KM ? make_sdesc(data_s, 16, 8 * RB, lt_for_pitch(RB)) : make_sdesc(data_s, 1024, MBs * 1024, LT_SW128);
  const uint64_t b_base = B0 ? make_sdesc(bmat_s, 16, 8 * 32, LT_SW32) : make_sdesc(bmat_s, 16, 16 * R, lt_for_pitch(2 * R));
  for (int t = 0; t < T; t++) {
    for (int p = 0; p < 2; p++) {
      for (int j = 0; j < NJ; j++) {
        const int ks = p * NSL + j;
        uint32_t aoff;
        if constexpr (KM) {
          const uint32_t colblk = R == 64 ? (uint32_t)((ks >> 2) * P::rows(SID) * 128) : 0u;
          aoff = colblk + (uint32_t)(t * 128 * RB) + (uint32_t)(32 * (R == 64 ? (ks & 3) : ks));
        } else {
          aoff = (uint32_t)((2 * ks * MBs + 2 * t) << 10);
        }
        const uint64_t ad = sdesc_add(a_base, aoff);
        for (int sp = 0; sp < P::NSET; sp++) {
          uint32_t boff;
          if constexpr (B0) {
            // duplicated-K blocks [-Fi', Fr', Fi']: forward real plane -> window 1, imag plane -> window 0
            boff = (uint32_t)(P::b0_off(sp) + (p == 0 ? 1 : 0) * 16 * 32);
          } else {
            const int w = INV ? (p == 0 ? 1 : 0) : (p == 0 ? 3 : 2);
            const int bj = SID == 0 ? (j % HS) : j;
            boff = (uint32_t)(P::slot_off(R, sp) + w * R * 2 * R + 32 * bj);
          }
          ops.mma(tmem + (uint32_t)(t * 2 * R), ad, sdesc_add(b_base, boff), idesc, (uint32_t)((p | j | sp) != 0));
        }
      }
    }
  }
}

// Twiddle exponent reduced to (-N/2, N/2] and turned into the argument of sincospi: angle = -2*pi*e/N.
template <int N>
SF_HD float tw_arg(int e) {
  e &= (N - 1);
  if (e > N / 2) e -= N;
  return -2.0f * (float)e / (float)N;
}

// ---------------------------------------------------------------------------------------------
// Epilogue for stage SID: one thread per TMEM lane (row r = t*128 + q*32 + lane of tile t).
// ---------------------------------------------------------------------------------------------
struct EpiArgs {
  uint32_t tmem;        // TMEM base of the group's accumulator slot
  const float* Kf;      // [H][N] complex fp32, digit order
  void* y;              // output base (TIO*)
  int B, H, cta;        // cta: the group index (pairs cta*G .. cta*G + G - 1)
  const uint8_t* kst;   // spectrum rows of channels khf, khf+1, ... staged by the loader warp, or null
  int khf;
  const float* en;      // the group's energy slots (its rows' output scales follow from them, pair_scales)
  // output stage: pair sg's output scales (pair_out_scales), kept across a thread's units of that pair
  mutable int sg = -1;
  mutable float so0 = 0.f, so1 = 0.f;
};

// 1/sqrt(R): the per-stage scale of a radix-R digit (the reference's 1/sqrt(R) per stage, total 1/N).
SF_HD constexpr float stage_scale(int R) { return R == 16 ? 0.25f : (R == 64 ? 0.125f : 0.17677669529663687f); }

// Spectrum values as the spectrum stage consumes them: per 16-byte piece (two complex values k0, k1 of
// Kf), {s*re(k0), s*re(k1), s*im(k0), s*im(k1)} with s = stage_scale of the spectrum stage's radix, so
// that the complex multiply runs on two elements per f32x2 operation and needs no separate scaling.
SF_HD void spec_piece(const float* raw4, float s, float* out4) {
  out4[0] = s * raw4[0];
  out4[1] = s * raw4[2];
  out4[2] = s * raw4[1];
  out4[3] = s * raw4[3];
}

// Byte offset of the 16-byte piece j (two complex values, in the spec_piece format) of 16-value chunk c of
// row rr in a staged spectrum row of a plan whose last radix is R (rows = N / R): [c][rr][piece ^ rr%8],
// so the 32 rows a warp reads hit 32 different bank groups.
template <int N, int R>
SF_HD uint32_t kstage_off(int rr, int c, int j) {
  return (uint32_t)((((c * (N / R) + rr) << 3) + (j ^ (rr & 7))) << 4);
}

// Number of 16-column chunks an epilogue thread reads per row in stage SID (the last inverse stage only
// needs time rows n0 < R0/2).
template <class P, int SID>
SF_HD constexpr int epi_chunks() {
  return SID == 2 * P::S - 1 ? (P::R0 / 2 < 16 ? 1 : P::R0 / 32) : P::rad(SID) / 16;
}

// Byte offsets of the 16-byte runs (m, k) and (m + 8, k) in an MN-major 128-B-swizzled operand (m % 8 == 0).
SF_HD void mn_off2(int m, int k, int MB, uint32_t* o0, uint32_t* o1) {
  const uint32_t kb = (uint32_t)((k >> 3) * MB) << 10;
  const uint32_t kr = (uint32_t)((k & 7) << 7), xk = (uint32_t)(k & 7);
  const uint32_t m8 = (uint32_t)(m >> 3), m8b = m8 + 1;
  *o0 = kb + kr + ((m8 >> 3) << 10) + (((m8 & 7) ^ xk) << 4);
  *o1 = kb + kr + ((m8b >> 3) << 10) + (((m8b & 7) ^ xk) << 4);
}

// Position of output element e (sequence-major over the group) in the swizzled fp32 staging of a
// 3-stage plan's output: the word index's low 5 bits are XOR-ed with bits 5..9, so the stride-R2 writes
// of a warp hit 32 different banks.
SF_HD uint32_t out_stage_word(int e) { return (uint32_t)(e ^ ((e >> 5) & 31)); }

// Per-thread indices of one epilogue unit: TMEM lane row r = t*128 + q*32 + lane of tile t, columns
// [16c, 16c + 16) of both the real and the imaginary half of the accumulator slot at `tmem`.
//   ta, tb   twiddle exponent e(col) = ta*col + tb of the four-step twiddle after this stage
//   m0, kre  first M row and real-plane K row of the next stage's operand written by this thread
//   vv       output position inside a sequence (last inverse stage)
struct EpiIdx {
  uint32_t taddr;
  int g, rr, c0, ta, tb, m0, kre, vv, r;
};

template <class P, int SID>
SF_HD EpiIdx epi_idx(uint32_t tmem, int t, int c, int q, int lane) {
  constexpr int S = P::S, R = P::rad(SID), N = P::N, RPP = N / R;   // rows per pair
  EpiIdx x;
  x.r = t * 128 + q * 32 + lane;
  x.g = x.r / RPP;
  x.rr = x.r - x.g * RPP;
  x.c0 = 16 * c;
  x.taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(t * 2 * R + x.c0);
  x.ta = x.tb = x.m0 = x.kre = x.vv = 0;
  const int g = x.g, rr = x.rr;
  if constexpr (SID == 0) {
    if constexpr (S == 2) { x.ta = rr; x.m0 = g * P::R0; x.kre = rr; }
    else {
      const int n1 = rr / P::R2, n2 = rr - n1 * P::R2;
      x.ta = rr; x.m0 = g * P::R0 * P::R2 + n2 * P::R0; x.kre = n1;
    }
  } else if constexpr (S == 3 && SID == 1) {
    const int n2 = rr / P::R0, k0 = rr - n2 * P::R0;
    x.ta = P::R0 * n2; x.m0 = g * P::R0 * P::R1 + k0 * P::R1; x.kre = n2;
  } else if constexpr (SID == S && S == 2) {
    x.ta = -rr; x.m0 = g * P::R1; x.kre = rr;
  } else if constexpr (SID == S && S == 3) {
    const int k0 = rr / P::R1, k1 = rr - k0 * P::R1;
    x.ta = -P::R0 * k1; x.m0 = g * P::R0 * P::R2 + k0 * P::R2; x.kre = k1;
  } else if constexpr (S == 3 && SID == S + 1) {
    const int k0 = rr / P::R2, n2 = rr - k0 * P::R2;
    x.ta = -k0 * P::R2; x.tb = -k0 * n2; x.m0 = g * P::R1 * P::R2 + n2 * P::R1; x.kre = k0;
  } else if constexpr (SID == 2 * S - 1) {
    if constexpr (S == 2) x.vv = rr;
    else { const int n2 = rr / P::R1, n1 = rr - n2 * P::R1; x.vv = n1 * P::R2 + n2; }
  }
  return x;
}

// Spectrum values of the 16 columns [c0, c0 + 16) of row rr for channel h, in the spec_piece format (eight
// pieces of four floats), from the loader's staged rows (stored in that format) when the group's channels
// are staged, else from Kf in global memory (converted here).  An empty pair slot (h < 0, past the last
// pair) reads any valid row; its outputs are never stored.
template <class P, int SID, class Ops>
SF_HD void load_spec(Ops& ops, const EpiArgs& ea, int h, int rr, int c0, float* kk) {
  constexpr int R = P::rad(SID), N = P::N;
  if (ea.kst) {
    const uint8_t* kb = ea.kst + (size_t)((h < 0 ? ea.khf : h) - ea.khf) * (N * 8);
    for (int j = 0; j < 8; j++) {
      float k4[4];
      ops.ldsK(kb + kstage_off<N, R>(rr, c0 >> 4, j), k4);
      kk[4 * j] = k4[0]; kk[4 * j + 1] = k4[1]; kk[4 * j + 2] = k4[2]; kk[4 * j + 3] = k4[3];
    }
  } else {
    const float* Kp = ea.Kf + 2 * ((long long)(h < 0 ? 0 : h) * N + (long long)rr * R + c0);
    for (int j = 0; j < 8; j++) {
      float k4[4];
      ops.ldK(Kp + 4 * j, k4);
      spec_piece(k4, stage_scale(R), kk + 4 * j);
    }
  }
}

// Second half of an epilogue unit, after its TMEM words have arrived: scale, twiddle (or spectrum
// multiply), round to fp16 and write the next stage's operand -- or, after the last stage, the outputs.
template <class P, class TIO, bool ACC16, int SID, class Ops>
SF_HD void epi_finish(Ops& ops, const EpiArgs& ea, const GroupPairs& gp, const EpiIdx& x, const uint32_t* raw_re,
                      const uint32_t* raw_im, const float* kk) {
  constexpr int S = P::S, R = P::rad(SID), N = P::N;
  constexpr bool OUT = (SID == 2 * S - 1), SPEC = (SID == S - 1);
  constexpr float SC = (R == 16) ? 0.25f : (R == 64 ? 0.125f : 0.17677669529663687f);
  const int g = x.g, c0 = x.c0, r = x.r;
  float a[16], b[16];
  for (int j = 0; j < 16; j++) { a[j] = ops.acc_val(raw_re[j]); b[j] = ops.acc_val(raw_im[j]); }

  if constexpr (OUT) {
    // each row's scale undoes its input scaling (pair_scales): a power of two, or 0 for an all-zero row
    if (g != ea.sg) {
      pair_out_scales<P, Shape<P, (int)sizeof(TIO)>::TWARPS * 32>(ea.en, g, &ea.so0, &ea.so1);
      ea.sg = g;
    }
    const float s0 = ea.so0 * SC, s1 = ea.so1 * SC;
    if constexpr (S == 2) {
      const PairInfo pi = gp.get(g, P::L);
      TIO* y = (TIO*)ea.y;
      constexpr int V0 = N / P::R0;
      for (int j = 0; j < 16; j++) {
        const int n0 = c0 + j;
        if (n0 < P::R0 / 2) {
          if (pi.off0 >= 0) ops.store1(y + pi.off0 + (long long)n0 * V0 + x.vv, a[j] * s0);
          if (pi.off1 >= 0) ops.store1(y + pi.off1 + (long long)n0 * V0 + x.vv, b[j] * s1);
        }
      }
    } else {
      // 3-stage plans: stage the pair's outputs in the (now free) data buffer; copied out coalesced
      constexpr int V0 = N / P::R0;
      for (int j = 0; j < 16; j++) {
        const int n0 = c0 + j;
        if (n0 < P::R0 / 2) {
          const int n = n0 * V0 + x.vv;
          ops.st4(out_stage_word(g * 2 * P::L + n) * 4, a[j] * s0);
          ops.st4(out_stage_word(g * 2 * P::L + P::L + n) * 4, b[j] * s1);
        }
      }
    }
    return;
  }

  uint32_t pr[8], pim[8];
  if constexpr (SPEC) {
    ops.cmul16(a, b, kk, pr, pim);   // (a + ib) x the scaled spectrum, rounded to fp16 pairs
    constexpr int RWS = P::rows(SID + 1);
    ops.st16(kmaj_data_off(r, c0, R, RWS), pr[0], pr[1], pr[2], pr[3]);
    ops.st16(kmaj_data_off(r, c0 + 8, R, RWS), pr[4], pr[5], pr[6], pr[7]);
    ops.st16(kmaj_data_off(r, R + c0, R, RWS), pim[0], pim[1], pim[2], pim[3]);
    ops.st16(kmaj_data_off(r, R + c0 + 8, R, RWS), pim[4], pim[5], pim[6], pim[7]);
  } else {
    float t0r, t0i, t8r, t8i, wr, wi;
    ops.tw(x.ta * c0 + x.tb, &t0r, &t0i);
    ops.tw(x.ta * (c0 + 8) + x.tb, &t8r, &t8i);
    ops.tw(x.ta, &wr, &wi);
    ops.twiddle16(a, b, t0r * SC, t0i * SC, t8r * SC, t8i * SC, wr, wi, pr, pim);
    constexpr int MBn = P::MB(SID + 1), Rn = P::rad(SID + 1);
    uint32_t o0, o1;
    mn_off2(x.m0 + c0, x.kre, MBn, &o0, &o1);
    constexpr uint32_t IMOFF = (uint32_t)(Rn / 8) * MBn * 1024;   // K-row Rn + kre is Rn/8 groups further
    ops.st16(o0, pr[0], pr[1], pr[2], pr[3]);
    ops.st16(o1, pr[4], pr[5], pr[6], pr[7]);
    ops.st16(o0 + IMOFF, pim[0], pim[1], pim[2], pim[3]);
    ops.st16(o1 + IMOFF, pim[4], pim[5], pim[6], pim[7]);
  }
}

// NU epilogue units of one thread (units u0, u0 + ustride, ...; unit u = tile u / C, chunk u % C): all
// their TMEM loads (and, in the spectrum stage, their spectrum loads) are issued before one wait, so
// their latencies overlap.
template <class P, class TIO, bool ACC16, int SID, int NU, class Ops>
SF_HD void epilogue_units(Ops& ops, const EpiArgs& ea, const GroupPairs& gp, int u0, int ustride, int q, int lane) {
  constexpr int C = epi_chunks<P, SID>(), R = P::rad(SID);
  constexpr bool SPEC = SID == P::S - 1;
  // spectrum loads ahead of the wait only where registers allow (4-warp plans: 184 per thread; the
  // 8-warp plans' ~95 would spill)
  constexpr bool EARLY = SPEC && P::W == 4;
  EpiIdx x[NU];
  uint32_t rre[NU][16], rim[NU][16];
  float kk[SPEC ? NU : 1][SPEC ? 32 : 1];
  for (int i = 0; i < NU; i++) {
    const int u = u0 + i * ustride, t = u / C, c = u - t * C;
    x[i] = epi_idx<P, SID>(ea.tmem, t, c, q, lane);
    ops.tmem_ld16(x[i].taddr, rre[i]);
    ops.tmem_ld16(x[i].taddr + (uint32_t)R, rim[i]);
    if constexpr (EARLY) load_spec<P, SID>(ops, ea, gp.get(x[i].g, P::L).h, x[i].rr, x[i].c0, kk[i]);
  }
  ops.tmem_wait();
  for (int i = 0; i < NU; i++) {
    if constexpr (SPEC && !EARLY) load_spec<P, SID>(ops, ea, gp.get(x[i].g, P::L).h, x[i].rr, x[i].c0, kk[i]);
    epi_finish<P, TIO, ACC16, SID>(ops, ea, gp, x[i], rre[i], rim[i], kk[SPEC ? i : 0]);
  }
}

// Spectrum stage of a 2-stage plan on a team with one warp per lane quarter: a pair has N / R1 <= 128 rows
// (a divisor of 128), so the warp's rows in tiles t and t + 1 have the same row index rr and read the same
// spectrum values whenever their pairs share a channel -- loaded once per chunk and channel (used by the
// 4-warp plans, whose register budget holds the values across tiles).
template <class P, class TIO, bool ACC16, int SID, class Ops>
SF_HD void epi_spec_shared(Ops& ops, const EpiArgs& ea, const GroupPairs& gp, int q, int lane) {
  constexpr int C = epi_chunks<P, SID>(), R = P::rad(SID), T = P::tiles(SID);
  static_assert(128 % (P::N / R) == 0, "a pair's rows divide a tile");
#pragma unroll 1
  for (int c = 0; c < C; c++) {
    float kk[32];
    int kh = -2;
#pragma unroll 1
    for (int t = 0; t < T; t++) {
      const EpiIdx x = epi_idx<P, SID>(ea.tmem, t, c, q, lane);
      uint32_t rre[16], rim[16];
      ops.tmem_ld16(x.taddr, rre);
      ops.tmem_ld16(x.taddr + (uint32_t)R, rim);
      const int h = gp.get(x.g, P::L).h;
      if (h != kh) {
        load_spec<P, SID>(ops, ea, h, x.rr, x.c0, kk);
        kh = h;
      }
      ops.tmem_wait();
      epi_finish<P, TIO, ACC16, SID>(ops, ea, gp, x, rre, rim, kk);
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Twiddle stages of 3-stage plans (every stage except the spectrum stage S - 1 and the output stage 2S - 1)
// through one runtime-parameterized epilogue (see shared_twiddle): their four index maps differ only in
// constants, so one copy of the code serves all of them (the kernel's warps hop between stages, and one copy
// per stage costs instruction-cache misses).
// With the pair-row index rr = hi * D + lo (lo < D):
//   twiddle exponent of column col: (a1 hi + a2 lo) col + c hi lo
//   next operand: M row g * MG + mh hi + ml lo + column, K row kh hi + kl lo
// ---------------------------------------------------------------------------------------------
struct TwParams {
  int R, T, c_shift, rpp_shift, d_shift;   // radix, tiles, log2(16-column chunks), log2(rows per pair), log2(D)
  int a1, a2, c, MG, mh, ml, kh, kl;
  int MBn;                           // M blocks of the next stage's operand
  uint32_t imoff;                    // byte distance of the next operand's imaginary K rows
  float sc;                          // 1/sqrt(R)
};

SF_HD constexpr int ilog2(int v) { return v <= 1 ? 0 : 1 + ilog2(v / 2); }

template <class P, int SID>
SF_HD constexpr TwParams tw_params() {
  constexpr int S = P::S, R = P::rad(SID), N = P::N;
  TwParams t{};
  t.R = R;
  t.T = P::tiles(SID);
  t.c_shift = ilog2(R / 16);
  t.rpp_shift = ilog2(N / R);
  t.MBn = P::MB(SID + 1);
  t.imoff = (uint32_t)(P::rad(SID + 1) / 8) * (uint32_t)P::MB(SID + 1) * 1024u;
  t.sc = stage_scale(R);
  if (SID == 0 && S == 2) {             // rr = n1: exponent rr k0, operand (g R0 + k0, n1)
    t.d_shift = 0; t.a1 = 1; t.MG = P::R0; t.kh = 1;
  } else if (SID == 0) {                // rr = n1 R2 + n2: exponent rr k0, operand (g R0 R2 + n2 R0 + k0, n1)
    t.d_shift = ilog2(P::R2); t.a1 = P::R2; t.a2 = 1; t.MG = P::R0 * P::R2; t.ml = P::R0; t.kh = 1;
  } else if (SID == 1 && S == 3) {      // rr = n2 R0 + k0: exponent R0 n2 k1, operand (g R0 R1 + k0 R1 + k1, n2)
    t.d_shift = ilog2(P::R0); t.a1 = P::R0; t.MG = P::R0 * P::R1; t.ml = P::R1; t.kh = 1;
  } else if (SID == S && S == 2) {      // rr = k0: exponent -k0 k1, operand (g R1 + n1, k0)
    t.d_shift = 0; t.a1 = -1; t.MG = P::R1; t.kh = 1;
  } else if (SID == S) {                // rr = k0 R1 + k1: exponent -R0 k1 k2, operand (g R0 R2 + k0 R2 + n2, k1)
    t.d_shift = ilog2(P::R1); t.a2 = -P::R0; t.MG = P::R0 * P::R2; t.mh = P::R2; t.kl = 1;
  } else {                              // SID S + 1, rr = k0 R2 + n2: exponent -k0 (R2 n1 + n2), operand (g R1 R2 + n2 R1 + n1, k0)
    t.d_shift = ilog2(P::R2); t.a1 = -P::R2; t.c = -1; t.MG = P::R1 * P::R2; t.ml = P::R1; t.kh = 1;
  }
  return t;
}

// NU units of a thread (units u0, u0 + ustride, ...) of a twiddle stage: TMEM loads of all of them first, then
// the twiddle, rounding and the next stage's operand.
template <class P, class TIO, bool ACC16, int NU, class Ops>
SF_HD void twiddle_units(Ops& ops, const EpiArgs& ea, const TwParams& tp, int u0, int ustride, int q, int lane) {
  uint32_t rre[NU][16], rim[NU][16];
  int c0[NU], ta[NU], tb[NU], m0[NU], kre[NU];
  for (int i = 0; i < NU; i++) {
    const int u = u0 + i * ustride, t = u >> tp.c_shift, c = u - (t << tp.c_shift);
    const int r = t * 128 + q * 32 + lane, g = r >> tp.rpp_shift, rr = r - (g << tp.rpp_shift);
    const int hi = rr >> tp.d_shift, lo = rr - (hi << tp.d_shift);
    c0[i] = 16 * c;
    ta[i] = tp.a1 * hi + tp.a2 * lo;
    tb[i] = tp.c * hi * lo;
    m0[i] = g * tp.MG + tp.mh * hi + tp.ml * lo;
    kre[i] = tp.kh * hi + tp.kl * lo;
    const uint32_t taddr = ea.tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(t * 2 * tp.R + c0[i]);
    ops.tmem_ld16(taddr, rre[i]);
    ops.tmem_ld16(taddr + (uint32_t)tp.R, rim[i]);
  }
  ops.tmem_wait();
  for (int i = 0; i < NU; i++) {
    float a[16], b[16];
    for (int j = 0; j < 16; j++) { a[j] = ops.acc_val(rre[i][j]); b[j] = ops.acc_val(rim[i][j]); }
    float t0r, t0i, t8r, t8i, wr, wi;
    ops.tw(ta[i] * c0[i] + tb[i], &t0r, &t0i);
    ops.tw(ta[i] * (c0[i] + 8) + tb[i], &t8r, &t8i);
    ops.tw(ta[i], &wr, &wi);
    uint32_t pr[8], pim[8];
    ops.twiddle16(a, b, t0r * tp.sc, t0i * tp.sc, t8r * tp.sc, t8i * tp.sc, wr, wi, pr, pim);
    uint32_t o0, o1;
    mn_off2(m0[i] + c0[i], kre[i], tp.MBn, &o0, &o1);
    ops.st16(o0, pr[0], pr[1], pr[2], pr[3]);
    ops.st16(o1, pr[4], pr[5], pr[6], pr[7]);
    ops.st16(o0 + tp.imoff, pim[0], pim[1], pim[2], pim[3]);
    ops.st16(o1 + tp.imoff, pim[4], pim[5], pim[6], pim[7]);
  }
}

// Whether a plan's twiddle stages share one runtime-parameterized epilogue: 3-stage plans with one warp per
// lane quarter in a team (several teams per CTA, each at a different stage); measured on B200: L = 4096
// (32x16x16, four teams) 5 % faster, the 3-stage plans with two or four warps per quarter 1-3 % slower, the
// 2-stage plans (two twiddle stages) unchanged or slower.
template <class P, class TIO>
SF_HD constexpr bool shared_twiddle() {
  return P::S == 3 && Shape<P, (int)sizeof(TIO)>::NWQ == 1;
}

// A thread's share of a twiddle stage (see epi_warp for the unit order).
template <class P, class TIO, bool ACC16, class Ops>
SF_HD void twiddle_stage(Ops& ops, const EpiArgs& ea, const TwParams& tp, int wi, int q, int lane) {
  constexpr int NWQ = Shape<P, (int)sizeof(TIO)>::NWQ;
  constexpr int NU = (NWQ == 2 && P::W == 4) ? 2 : 1;
  const int U = tp.T << tp.c_shift;
  int u = wi;
  if constexpr (NU == 2) {
#pragma unroll 1
    for (; u + NWQ < U; u += 2 * NWQ) twiddle_units<P, TIO, ACC16, 2>(ops, ea, tp, u, NWQ, q, lane);
  }
#pragma unroll 1
  for (; u < U; u += NWQ) twiddle_units<P, TIO, ACC16, 1>(ops, ea, tp, u, NWQ, q, lane);
}

// The units of stage SID that one thread handles: its warp covers TMEM lane quarter q (warp % 4) and,
// being warp wi of the team's NWQ warps on that quarter, units wi, wi + NWQ, ...  With two warps per
// quarter on a 4-warp plan (registers to spare), units are taken in pairs so that two units' TMEM loads
// are in flight together.
template <class P, class TIO, bool ACC16, int SID, class Ops>
SF_HD void epi_warp(Ops& ops, const EpiArgs& ea, const GroupPairs& gp, int wi, int q, int lane) {
  if constexpr (shared_twiddle<P, TIO>() && SID != P::S - 1 && SID != 2 * P::S - 1) {
    constexpr TwParams tp = tw_params<P, SID>();
    twiddle_stage<P, TIO, ACC16>(ops, ea, tp, wi, q, lane);
    return;
  }
  constexpr int NWQ = Shape<P, (int)sizeof(TIO)>::NWQ;
  constexpr int C = epi_chunks<P, SID>(), U = P::tiles(SID) * C;
  constexpr bool SPEC = SID == P::S - 1;
  constexpr int NU = (NWQ == 2 && P::W == 4 && !SPEC && U % (2 * NWQ) == 0) ? 2 : 1;
  if constexpr (SPEC && P::S == 2 && NWQ == 1 && P::W == 4) {
    epi_spec_shared<P, TIO, ACC16, SID>(ops, ea, gp, q, lane);
  } else if constexpr (U % (NU * NWQ) == 0) {
#pragma unroll 1
    for (int i = 0; i < U / NWQ; i += NU) epilogue_units<P, TIO, ACC16, SID, NU>(ops, ea, gp, wi + i * NWQ, NWQ, q, lane);
  } else {
#pragma unroll 1
    for (int u = wi; u < U; u += NWQ) epilogue_units<P, TIO, ACC16, SID, 1>(ops, ea, gp, u, NWQ, q, lane);
  }
}

// Copy-out of a 3-stage plan's staged outputs (after every epilogue thread has staged its values):
// thread i moves 4 consecutive elements of the group's 2G sequences to y with one 16- or 8-byte store.
template <class P, class TIO, class Ops>
SF_HD void copy_out_staged(Ops& ops, const EpiArgs& ea, const GroupPairs& gp, int tid, int nthreads) {
  TIO* y = (TIO*)ea.y;
  const int total = P::G * 2 * P::L;
  for (int e = tid * 4; e < total; e += nthreads * 4) {
    const int seq = e / P::L, n = e - seq * P::L;
    const PairInfo pi = gp.get(seq >> 1, P::L);
    const long long off = (seq & 1) ? pi.off1 : pi.off0;
    float v[4];
    const uint32_t w = out_stage_word(e);            // e % 4 == 0: the 4 words share one XOR value
    ops.ld4_staged((w & ~3u) * 4, (w ^ (uint32_t)e) & 3u, v);
    if (off >= 0) ops.store4(y + off + n, v);
  }
}

// ---------------------------------------------------------------------------------------------
// Partitioned convolution of composite plans (L = P * Lb, blocks of the block plan's length Lb = P::L)
//
// The caller's [B][Hb][L] arrays are read as [B][Hb * P][Lb]: row (b, h) block q is "channel" h' = h * P + q of
// length Lb, so the kernel's pairs, groups and offsets apply unchanged.  With U_q the spectrum of input block q
// (zero-padded to N = 2 Lb) and K'_d the spectrum of the filter segment kw_d[n] = k[d Lb + n] (n < Lb),
// kw_d[Lb + m] = k[(d - 1) Lb + m] (m < Lb, zero for d = 0), output block p is the first Lb outputs of the
// inverse transform of W_p = sum_{q <= p} U_q K'_{p - q}: K'_d = K_d + (-1)^f K_{d-1} folds the second half of
// block p - 1's linear convolution (a shift by N / 2 is a sign flip of the odd frequencies) into block p.
//   forward launch:  conversion and stages 0 .. S-1 of every (pair, block); the last forward stage stores the
//                    pair's spectrum (x its 1/sqrt(R) stage scale) to Z [Hb * P][PB][N] (complex fp32, digit
//                    order) instead of multiplying it by a filter spectrum;
//   spectrum sums:   a streaming kernel (blocks.cu) replaces every pair's Z_p by W_p = sum_{q <= p} Z_q K'_{p-q}
//                    in place (the spectrum multiply of the single-pass kernel, extended over the blocks);
//   inverse launch:  the operand of stage S from W_p, then stages S .. 2S-1 and the outputs of block p.
// Both launches scale each row by the power of two that its energy over the whole row gives (pair_scales), so
// that every block of a row carries the same scale and the sum over blocks stays consistent; the energies come
// from a separate pass over u, normalised to Lb values.
// ---------------------------------------------------------------------------------------------
struct BlockArgs {
  float* Z;           // [Hb * P][PB][N] complex pair spectra of the input blocks
  const float* En;    // [B * Hb] row energies (sum of squares over the row x Lb / L)
  int lgP;            // log2 of the block count P
  int Hb;             // channels of the caller's arrays
};

// The group's energy slots from the row energies (slot 0 of each sequence holds its row's energy, the others
// zero), lanes i0, i0 + istep, ... of the caller; absent sequences have energy 0.
template <class P, int NT>
SF_HD void fill_energies(float* en, const BlockArgs& ba, const GroupPairs& gp, int i0, int istep) {
  using EN = Energy<P, NT>;
  constexpr int LGL = ilog2(P::L);
  for (int i = i0; i < EN::SLOTS; i += istep) {
    const int seq = i / EN::SPS, slot = i - seq * EN::SPS;
    float e = 0.f;
    if (slot == 0) {
      const PairInfo pi = gp.get(seq >> 1, P::L);
      const long long off = (seq & 1) ? pi.off1 : pi.off0;
      if (off >= 0) e = ba.En[off >> (LGL + ba.lgP)];
    }
    en[i] = e;
  }
}

// Forward launch, after the last forward stage: the pair spectra of the group's units to Z.
template <class P, class TIO, class Ops>
SF_HD void spec_store_units(Ops& ops, const EpiArgs& ea, const BlockArgs& ba, const GroupPairs& gp, int wi, int q,
                            int lane) {
  constexpr int SID = P::S - 1, C = epi_chunks<P, SID>(), R = P::rad(SID), U = P::tiles(SID) * C, N = P::N;
  constexpr int NWQ = Shape<P, (int)sizeof(TIO)>::NWQ;
  constexpr float SC = stage_scale(R);
#pragma unroll 1
  for (int u = wi; u < U; u += NWQ) {
    const int t = u / C, c = u - t * C;
    const EpiIdx x = epi_idx<P, SID>(ea.tmem, t, c, q, lane);
    uint32_t rre[16], rim[16];
    ops.tmem_ld16(x.taddr, rre);
    ops.tmem_ld16(x.taddr + (uint32_t)R, rim);
    ops.tmem_wait();
    const PairInfo pi = gp.get(x.g, P::L);
    if (pi.h < 0) continue;
    float* zp = ba.Z + 2 * (((long long)pi.h * gp.PB + pi.j) * N + (long long)x.rr * R + x.c0);
    for (int j = 0; j < 16; j += 2) {
      const float v[4] = {ops.acc_val(rre[j]) * SC, ops.acc_val(rim[j]) * SC, ops.acc_val(rre[j + 1]) * SC,
                          ops.acc_val(rim[j + 1]) * SC};
      ops.stZ(zp + 2 * j, v);
    }
  }
}

// Inverse launch, in place of the conversion: the A operand of stage S (the layout the spectrum stage's
// epilogue writes) from each unit's 16 values of the summed spectrum W_p (held in Z's slot of block p), in two
// runs of eight.
template <class P, class TIO, class Ops>
SF_HD void spec_load_units(Ops& ops, const BlockArgs& ba, const GroupPairs& gp, int wi, int q, int lane) {
  constexpr int SID = P::S - 1, C = epi_chunks<P, SID>(), R = P::rad(SID), U = P::tiles(SID) * C, N = P::N;
  constexpr int NWQ = Shape<P, (int)sizeof(TIO)>::NWQ, RWS = P::rows(SID + 1);
#pragma unroll 1
  for (int u = wi; u < U; u += NWQ) {
    const int t = u / C, c = u - t * C;
    const EpiIdx x = epi_idx<P, SID>(0u, t, c, q, lane);
    const PairInfo pi = gp.get(x.g, P::L);
    const int hb = pi.h >> ba.lgP, pb = pi.h - (hb << ba.lgP);
#pragma unroll 1
    for (int half = 0; half < 2; half++) {
      float ar[8], ai[8];
      for (int e = 0; e < 8; e++) ar[e] = ai[e] = 0.f;
      const long long pos = (long long)x.rr * R + x.c0 + 8 * half;
      if (pi.h >= 0) {
        const float* zp = ba.Z + 2 * ((((long long)(hb << ba.lgP) + pb) * gp.PB + pi.j) * N + pos);
        for (int e = 0; e < 4; e++) {
          float z4[4];
          ops.ldZ(zp + 4 * e, z4);
          ar[2 * e] = z4[0]; ai[2 * e] = z4[1]; ar[2 * e + 1] = z4[2]; ai[2 * e + 1] = z4[3];
        }
      }
      uint32_t pr[4], pim[4];
      for (int p = 0; p < 4; p++) {
        pr[p] = ops.pack2(ar[2 * p], ar[2 * p + 1]);
        pim[p] = ops.pack2(ai[2 * p], ai[2 * p + 1]);
      }
      ops.st16(kmaj_data_off(x.r, x.c0 + 8 * half, R, RWS), pr[0], pr[1], pr[2], pr[3]);
      ops.st16(kmaj_data_off(x.r, R + x.c0 + 8 * half, R, RWS), pim[0], pim[1], pim[2], pim[3]);
    }
  }
}

// ---------------------------------------------------------------------------------------------
// DFT-matrix region image (identical for the cached table and the in-kernel "legacy" build)
// ---------------------------------------------------------------------------------------------
// Calls emit(byte_off, radix, phase_index q, which, set) for every fp16 entry of the region;
// `which`: 0 -> cos(2*pi*q/R), 1 -> -sin(2*pi*q/R), 2 -> +sin(2*pi*q/R); `set` 0 = hi, 1 = lo.
#ifdef __CUDACC__
#pragma nv_exec_check_disable
#endif
template <class P, class Emit>
SF_HD void for_each_bmat_entry(Emit& emit, int tid, int nthreads) {
  for (int set = 0; set < P::NSET; set++) {
    for (int rq = 16; rq <= 64; rq <<= 1) {
      if (!P::uses(rq)) continue;
      const int base = P::slot_off(rq, set), total = 5 * rq * rq;
      for (int i = tid; i < total; i += nthreads) {
        const int row = i / rq, k = i - row * rq, b = row / rq, n = row - b * rq;
        int q, which;
        block_entry(b, n, k, rq, &q, &which);
        emit(base + (int)km_off(row, k, 2 * rq), rq, q, which, set);
      }
    }
    if (P::R0 == 16) {
      // first-stage blocks [-Fi', Fr', Fi'] with K duplicated: column k uses input index k % 8
      const int base = P::b0_off(set);
      for (int i = tid; i < 3 * 16 * 16; i += nthreads) {
        const int row = i / 16, k = i - row * 16, b = row / 16, n = row - b * 16;
        const int q = (n * (k & 7)) % 16, which = b == 1 ? 0 : (b == 0 ? 2 : 1);
        emit(base + (int)km_off(row, k, 32), 16, q, which, set);
      }
    }
  }
}

}  // namespace sffft
