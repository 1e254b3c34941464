// Compile-time plan math and tcgen05 shared-memory layouts for the fused causal convolution.
//
// A plan factors the zero-padded transform size N = 2L as N = R0*R1(*R2) with radices 16/32/64,
// exactly like the reference's Plan<R0,R1,R2> (sfFFT src/sffft.cu:92-104): stage j runs a DFT of
// size R(j) along digit j; the forward result sits in "digit order", position
//   p = k0*R1*R2 + k1*R2 + k2  holding frequency  k = k0 + R0*k1 + R0*R1*k2
// (the order permuteK produces, src/sffft.cu:283-288).  Every stage is scaled by 1/sqrt(R), so the
// forward+inverse pair is normalised by 1/N (src/sffft.cu:146,203).
//
// B200 layout of one CTA (this file only describes it; the kernel lives in fused_conv.cuh):
//   * G "pairs" per CTA.  A pair is two batch elements b=2j, 2j+1 of one channel h, packed as one
//     complex sequence z = u[2j] + i*u[2j+1]; the filter is real, so conv(z,k) = conv(u0,k) + i*conv(u1,k)
//     and one complex transform serves two real sequences.
//   * Each stage is one real GEMM per 128-row tile on tcgen05:  D[m, 0:2R] = [Zr | Zi](m, 0:2R) x Bwin,
//     rows m = the length-R vectors of that stage (all pairs of the CTA), D in TMEM (fp32 or fp16).
//   * A operands live in one data buffer (4*N*G bytes, rewritten in place by each epilogue) in the
//     canonical MN-major 128-byte-swizzled layout, except the inverse of the last digit, which uses the
//     same rows as the forward last digit and is K-major (each epilogue thread owns its row).
//   * B operands are the DFT matrices in K-major swizzled layouts, five R x R blocks
//     [Fi, Fr, -Fi, Fr, Fi]; the four 2R-row windows starting at blocks 0..3 are the real forms of
//     inverse-imag, inverse-real, forward-imag and forward-real input planes.
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define SF_HD __host__ __device__ __forceinline__
#else
#define SF_HD inline
#endif

namespace sffft {

SF_HD constexpr int cmax(int a, int b) { return a > b ? a : b; }
SF_HD constexpr int pow2ceil(int v) { int p = 1; while (p < v) p <<= 1; return p; }

// ---------------------------------------------------------------------------------------------
// Canonical UMMA shared-memory layouts for 16-bit elements (byte offsets from a 1024-B aligned base)
// ---------------------------------------------------------------------------------------------

// MN-major, 128-byte swizzle.  A K-row holds 64 consecutive M elements (128 B); 8 K-rows form a
// 1024-B atom; atom (m/64, k/8) sits at ((k/8)*MB + m/64)*1024.  Descriptor: LBO = 1024 (stride
// between 64-element M blocks), SBO = MB*1024 (stride between 8-row K groups).
SF_HD uint32_t mn_off(int m, int k, int MB) {
  return ((uint32_t)((k >> 3) * MB + (m >> 6)) << 10) + (uint32_t)((k & 7) << 7) +
         (uint32_t)(((((m >> 3) & 7) ^ (k & 7))) << 4) + (uint32_t)((m & 7) << 1);
}

// K-major with row pitch RB in {32, 64, 128} bytes and swizzle width equal to RB; rows are
// contiguous so 8 rows form one swizzle atom (8*RB bytes).  Descriptor: SBO = 8*RB.
SF_HD uint32_t km_off(int r, int k, int RB) {
  const int sw = RB == 128 ? (r & 7) : RB == 64 ? ((r & 7) >> 1) : ((r & 7) >> 2);
  return (uint32_t)(r * RB) + (uint32_t)(((((k * 2) >> 4) ^ sw)) << 4) + (uint32_t)((k & 7) << 1);
}

// tcgen05 layout-type codes (smem descriptor bits 61..63)
enum : int { LT_NONE = 0, LT_SW128 = 2, LT_SW64 = 4, LT_SW32 = 6 };
SF_HD constexpr int lt_for_pitch(int RB) { return RB == 128 ? LT_SW128 : RB == 64 ? LT_SW64 : LT_SW32; }

// Shared-memory matrix descriptor (tcgen05 format, version 1).
SF_HD uint64_t make_sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo, int layout) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}

// Instruction descriptor for tcgen05.mma kind::f16 with f16 A/B.
SF_HD constexpr uint32_t make_idesc(int M, int N, bool d_f32, bool a_mn, bool b_mn) {
  return ((d_f32 ? 1u : 0u) << 4) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---------------------------------------------------------------------------------------------
// Plan
// ---------------------------------------------------------------------------------------------
// MS_: the most group slots (and teams) per CTA.  The catalog plans use 4; small launches, with at most one
// or two groups per SM, run variants with 1 or 2 slots whose teams are 4x or 2x wider (shorter chains).
// SPLIT_: three-stage plans hold their DFT matrices as fp16 hi + lo (IoPlan clears it for bf16 I/O).
template <int R0_, int R1_, int R2_, int G_, int W_, int MS_ = 4, bool SPLIT_ = true>
struct Plan {
  static constexpr int R0 = R0_, R1 = R1_, R2 = R2_, G = G_, W = W_, MS = MS_;
  static constexpr int S = R2_ > 1 ? 3 : 2;
  static constexpr int N = R0 * R1 * R2, L = N / 2, NT = 32 * W;
  static constexpr int RL = S == 3 ? R2 : R1;          // radix of the last (contiguous) digit
  static constexpr bool FSPLIT = S == 3 && SPLIT_;      // DFT matrices as fp16 hi + lo (accuracy)
  static constexpr int NSET = FSPLIT ? 2 : 1;

  SF_HD static constexpr int R(int j) { return j == 0 ? R0 : (j == 1 ? R1 : R2); }
  SF_HD static constexpr int digit(int sid) { return sid < S ? sid : 2 * S - 1 - sid; }
  SF_HD static constexpr bool inv(int sid) { return sid >= S; }
  SF_HD static constexpr int rad(int sid) { return R(digit(sid)); }
  SF_HD static constexpr int rows(int sid) { return G * (N / rad(sid)); }   // GEMM M for this stage
  SF_HD static constexpr int tiles(int sid) { return rows(sid) / 128; }
  SF_HD static constexpr int cols(int sid) { return tiles(sid) * 2 * rad(sid); }
  SF_HD static constexpr bool kmajor(int sid) { return sid == S; }
  SF_HD static constexpr int MB(int sid) { return rows(sid) / 64; }

  static constexpr int max_cols() {
    int c = 0;
    for (int s = 0; s < 2 * S; s++) c = cmax(c, cols(s));
    return c;
  }
  static constexpr int TMEM_COLS = cmax(32, pow2ceil(max_cols()));
  static constexpr int DATA_BYTES = 4 * N * G;

  // DFT-matrix region: one slot per distinct radix (five R x R blocks, NSET sets), plus the
  // duplicated-K first-stage matrix when R0 == 16 (three 16 x 16 blocks, NSET sets).
  SF_HD static constexpr bool uses(int r) { return R0 == r || R1 == r || R2 == r; }
  SF_HD static constexpr int slot_bytes(int r) { return ((5 * r * 2 * r + 1023) / 1024) * 1024; }
  SF_HD static constexpr int slot_off(int r, int set) {
    int off = 0;
    for (int q = 16; q <= 64; q <<= 1) {
      if (!uses(q)) continue;
      for (int s = 0; s < NSET; s++) {
        if (q == r && s == set) return off;
        off += slot_bytes(q);
      }
    }
    return off;
  }
  static constexpr int B0_BYTES = 2048;   // 3 blocks x 16 rows x 32 B = 1536, padded
  SF_HD static constexpr int b0_off(int set) { return slot_off(128, 0) + set * B0_BYTES; }
  static constexpr int BMAT_BYTES = slot_off(128, 0) + (R0 == 16 ? NSET * B0_BYTES : 0);
  static constexpr int SMEM_BYTES = DATA_BYTES + BMAT_BYTES + 64 + 1024;   // + barrier, tmem slot, align

  static_assert(N % 256 == 0, "N must be >= 256");
  static_assert((R0 == 16 || R0 == 32 || R0 == 64) && (R1 == 16 || R1 == 32 || R1 == 64) &&
                (R2 == 1 || R2 == 16 || R2 == 32 || R2 == 64), "radices must be 16/32/64");
  static_assert(W == 4 || W == 8, "4 or 8 warps");
};

// The plan a kernel with I/O element size SIO runs.  The hi + lo split of three-stage plans' DFT matrices keeps
// fp32 I/O within its tolerance (relative L2 3.5e-4 with it, 4.3-5.0e-4 without, against 5e-4); bf16 I/O is
// rounded to bf16 at the output, which the split does not change (1.69e-3 with, 1.71e-3 without at L = 4096,
// against 3e-3), so its kernels run one fp16 set: half the MMAs of every stage and half the matrix bytes.
template <class P, int SIO>
struct IoPlanT {
  using type = P;
};
template <int R0, int R1, int R2, int G, int W, int MS>
struct IoPlanT<Plan<R0, R1, R2, G, W, MS, true>, 2> {
  using type = Plan<R0, R1, R2, G, W, MS, (R2 == 1)>;   // two-stage plans: the same type (no split either way)
};
template <class P, int SIO>
using IoPlan = typename IoPlanT<P, SIO>::type;

// Resources of the persistent kernel for plan P and I/O element size SIO:
//   1 L2-prefetch warp (a few groups ahead of the conversions), 1 MMA warp, 1 spectrum-loader warp, and
//   WC = 2W compute warps split into NTEAM teams of TWARPS warps (a multiple of 4, so a team covers all
//   four TMEM lane quarters).
//   NS slots: a slot holds one group in flight (a data buffer and a TMEM accumulator region).  Team t
//   owns slots t*NST .. t*NST + NST - 1 and steps through its groups' tasks on its own (it reads its
//   groups' input straight from global memory); the MMA warp serves whichever slot is ready, so one
//   team's waits are filled by another team's work.
//   Shared memory after the DFT matrices and the NS data buffers: the spectrum staging area (KSLOT slots
//   of KC channel rows).
// Slot policy: one slot per team of four compute warps (a team that alternates between two slots of its
// own loses more to lockstep than it gains), at most SFFFT_MAX_SLOTS, as many as TMEM and shared memory hold.
#ifndef SFFFT_MAX_SLOTS
#define SFFFT_MAX_SLOTS 4
#endif
#ifndef SFFFT_MAX_TEAMS
#define SFFFT_MAX_TEAMS 4
#endif
template <class P, int SIO>
struct Shape {
  static constexpr int WC = 2 * P::W;
  static constexpr int CW0 = 3;                                     // first compute warp
  static constexpr int NT = 32 * (WC + CW0);
  static constexpr int SEQB = P::L * SIO;                           // input bytes per sequence
  static constexpr int TW_BYTES = ((64 + P::N / 64) * 8 + 127) / 128 * 128;   // two-level twiddle table
  // per slot and round parity: the conversion's energy slots of the group's 2G sequences, one per warp of a
  // sequence (at most max(2G, 2W) floats for any team size)
  static constexpr int EN_STRIDE_MAX = 2 * P::G > 2 * P::W ? 2 * P::G : 2 * P::W;
  static constexpr int EN_BYTES_MAX = (4 * 2 * EN_STRIDE_MAX * 4 + 127) / 128 * 128;   // for up to 4 slots
  static constexpr int CAP = 227 * 1024 - 1024 - 512 - TW_BYTES - EN_BYTES_MAX;   // dynamic smem minus align
                                                                                // slack, barriers, energies
  static constexpr bool fits(int ns) {
    return ns * P::TMEM_COLS <= 512 && P::BMAT_BYTES + ns * P::DATA_BYTES <= CAP;
  }
  static constexpr int SLOTCAP = SFFFT_MAX_SLOTS < P::MS ? SFFFT_MAX_SLOTS : P::MS;
  static constexpr int NSMAX = WC / 4 < SLOTCAP ? WC / 4 : SLOTCAP;
  static constexpr int NS = (NSMAX >= 4 && fits(4)) ? 4 : ((NSMAX >= 2 && fits(2)) ? 2 : 1);
  static constexpr int NSLOT = NS;
  static constexpr int TMAXW = WC / 4 < SFFFT_MAX_TEAMS ? WC / 4 : SFFFT_MAX_TEAMS;
  static constexpr int NTEAM = NS < TMAXW ? NS : TMAXW;             // NS, WC / 4 and the cap are powers of two
  static constexpr int NST = NS / NTEAM;                            // slots per team
  static constexpr int TWARPS = WC / NTEAM;                         // warps per team
  static constexpr int NWQ = TWARPS / 4;                            // a team's warps per TMEM lane quarter
  static constexpr int NB = P::W == 4 ? 4 : 2;                      // conversion steps whose loads overlap
  // L2 prefetch distance in groups: NS + 1, but at most kPrefetchBytes of input and spectrum rows ahead of
  // the conversions per CTA (about 24 MB over 148 CTAs).  Prefetching further ahead at long lengths evicts
  // the spectrum rows and outputs of the groups in flight (measured: one group ahead is 2-4 % faster than
  // NS + 1 at L = 8192 and 16384, two ahead 5 % faster at L = 2048, no change at L <= 1024).
  static constexpr int kPrefetchBytes = 160 * 1024;
  static constexpr int GROUP_L2_BYTES = 2 * P::G * SEQB + P::N * 8;
  static constexpr int PD = kPrefetchBytes / GROUP_L2_BYTES < 1 ? 1
                            : (kPrefetchBytes / GROUP_L2_BYTES > NS + 1 ? NS + 1 : kPrefetchBytes / GROUP_L2_BYTES);
  static constexpr int DATA_OFF = P::BMAT_BYTES;
  static constexpr int K_OFF = DATA_OFF + NS * P::DATA_BYTES;
  static constexpr int FREE = CAP - K_OFF;
  // spectrum staging: KSLOT slots of KC channel rows (N complex fp32 each), filled by the loader warp in a
  // swizzled [chunk][row][16 B ^ row%8] order; groups spanning more than KC channels read Kf from global.
  // A single slot serialises several teams' spectrum stages (measured slower than global reads), so it
  // is used only by a CTA with one team.
  static constexpr int KROW = P::N * 8;
  static constexpr int KSLOT = FREE >= 2 * KROW ? 2 : ((FREE >= KROW && NTEAM == 1) ? 1 : 0);
  static constexpr int KX = KSLOT > 0 ? FREE / (KSLOT * KROW) : 0;
  static constexpr int KC = KSLOT == 0 ? 0 : (KX < P::G ? KX : P::G);
  static constexpr int KBYTES = KSLOT * KC * KROW;
  static constexpr int TW_OFF = K_OFF + KBYTES;
  static constexpr int BAR_OFF = TW_OFF + TW_BYTES;
  static constexpr int EN_OFF = BAR_OFF + 512;
  static constexpr int EN_STRIDE_RAW = 2 * P::G * ((TWARPS * 32 / (2 * P::G)) / 32 > 1 ? (TWARPS * 32 / (2 * P::G)) / 32 : 1);
  static constexpr int EN_STRIDE = EN_STRIDE_RAW;
  static constexpr int EN_BYTES = (NS * 2 * EN_STRIDE * 4 + 127) / 128 * 128;
  static constexpr int SMEM = EN_OFF + EN_BYTES + 1024;
  static constexpr int TMEM_ALLOC = pow2ceil(cmax(32, NS * P::TMEM_COLS));
  static constexpr int TPG = 2 * P::S + 1;                          // tasks per group: convert + 2S epilogues
  // 8-byte words from BAR_OFF: a_ready[NS], mma_done[NS], k_full[2], k_empty[2], TMEM base, abort flag,
  // first staged channel per spectrum slot[2], team_done[NTEAM], bmat_full, then ints: spectrum slot stamps[2],
  // the count of converted groups and the stage-repeat flags[NS]
  static constexpr int NBARW = 2 * NS + 4 + 3 + NTEAM + 1 + (3 + NS + 1) / 2;
  static_assert(NBARW <= 64, "barrier area");
  static_assert(NS % NTEAM == 0 && WC % (4 * NTEAM) == 0, "teams");
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(SEQB % 16 == 0, "sequences are whole 16-byte runs");
};

// Row pitch of the K-major A operand of the inverse last-digit stage (re | im halves of a row).
SF_HD constexpr int kmaj_data_pitch(int R) { return 4 * R > 128 ? 128 : 4 * R; }

// Byte offset of element (row r, k) of the K-major data operand with `rows` rows and radix R.
// R = 64 rows (256 B) are split into two 128-B column blocks of rows*128 bytes each.
SF_HD uint32_t kmaj_data_off(int r, int k, int R, int rows) {
  if (R == 64) return (uint32_t)((k >> 6) * rows * 128) + km_off(r, k & 63, 128);
  return km_off(r, k, 4 * R);
}

// Value of DFT-matrix block b (0..4 = Fi, Fr, -Fi, Fr, Fi) at (n, k) for radix R, as a multiple of
// 2*pi/R phase index and a selector: returns (phase index q = n*k mod R, which = 0 cos, 1 -sin, 2 +sin)
SF_HD void block_entry(int b, int n, int k, int R, int* q, int* which) {
  *q = (n * k) % R;
  *which = (b == 1 || b == 3) ? 0 : (b == 2 ? 2 : 1);
}

}  // namespace sffft
