// The fused causal-convolution kernel for sm_100a (persistent, warp-specialised).
//
// Replaces the reference kernel fftconv<Plan,W,TIO,TAcc,CACHED> (sfFFT src/sffft.cu:243-280): the same
// four-step transform, spectrum multiply and inverse, but one CTA per SM loops over "groups" of G pairs of
// sequences (two batch elements of one channel per pair) with four roles:
//
//   warp 0 (prefetch)  brings each group's input sequences and spectrum rows into L2 (bulk prefetches), a
//                      few groups ahead of the conversions;
//   warp 1 (MMA)       allocates TMEM and issues each stage's tcgen05.mma's as soon as a team has written
//                      that slot's A operand, then commits to the slot's "stage done" mbarrier;
//   warp 2 (spectrum)  stages each group's spectrum rows in shared memory, swizzled for the epilogue;
//   warps 3.. (compute) in teams of four or more (one warp per TMEM lane quarter): each team owns slots
//                      (a data buffer and a TMEM region each, one group in flight per slot), converts its
//                      groups' u (read straight from global memory) to the first-stage operand (fp16 hi +
//                      lo) and runs every stage's epilogue: TMEM -> registers -> twiddle / spectrum / scale
//                      -> the next stage's operand in shared memory (or y in global memory).
//
// Teams run independently, so one team's waits on its MMAs are covered by the others' epilogues.  Every
// wait is bounded: after kWaitLimitNs a role records SFFFT_ERR_TIMEOUT in *status, raises a shared abort
// flag that ends the other roles' loops, and the CTA frees its TMEM.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "stages.h"
#include "status.h"
#include "tc.cuh"

namespace sffft {

constexpr unsigned long long kWaitLimitNs = 1000000000ull;   // default: 1 s per barrier phase

// The launch's wait limit (ConvParams::wait_ns, or the default), set by thread 0 before the first block barrier.
static __shared__ unsigned long long s_wait_ns;

__device__ __forceinline__ float bf16_bits_to_float(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

typedef unsigned long long u64;
__device__ __forceinline__ u64 pk2(float lo, float hi) {
  u64 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void up2(u64 v, float& lo, float& hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
// Blackwell packed fp32 arithmetic: two independent IEEE fp32 lanes per instruction.
__device__ __forceinline__ u64 fma2(u64 a, u64 b, u64 c) {
  u64 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ u64 mul2(u64 a, u64 b) {
  u64 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Shared memory is addressed through 32-bit shared-window addresses (st.shared / ld.shared): the dynamic
// shared-memory base is aligned through an integer cast, so pointers derived from it are generic, and generic
// accesses cost 64-bit address arithmetic and registers in every epilogue unit (measured: 6 % fewer warp
// instructions and 1-7 % faster launches with shared-window addresses).
struct DevOps {
  uint32_t sm;      // shared-window address of the data buffer the epilogue / conversion writes
  bool acc16;
  uint32_t tw_lo;   // shared-window address of w_N^e, e in [0, 64) (float2 each)
  uint32_t tw_hi;   // of w_N^(64 h), h in [0, N/64)
  int n_tw;         // transform size N
  __device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    mma_f16_ss(d, a, b, idesc, acc);
  }
  __device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) { sffft::tmem_ld16(taddr, r); }
  __device__ __forceinline__ void tmem_wait() { tmem_wait_ld(); }
  __device__ __forceinline__ void st16(uint32_t off, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sm + off), "r"(a), "r"(b), "r"(c), "r"(d));
  }
  __device__ __forceinline__ void sincospi(float x, float* s, float* c) { sincospif(x, s, c); }
  __device__ __forceinline__ uint32_t pack2(float lo, float hi) const {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ float lo16f(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu))); }
  __device__ __forceinline__ float hi16f(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }
  __device__ __forceinline__ float acc_val(uint32_t w) { return acc16 ? lo16f(w) : __uint_as_float(w); }
  __device__ __forceinline__ void ldsK(const void* p, float (&k)[4]) {
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(k[0]), "=f"(k[1]), "=f"(k[2]), "=f"(k[3])
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
  }
  __device__ __forceinline__ void ldK(const float* p, float (&k)[4]) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(p));
    k[0] = v.x; k[1] = v.y; k[2] = v.z; k[3] = v.w;
  }
  // pair spectra of composite plans: written by the forward launch, read (only) by the inverse launch
  __device__ __forceinline__ void ldZ(const float* p, float (&z)[4]) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(p));
    z[0] = v.x; z[1] = v.y; z[2] = v.z; z[3] = v.w;
  }
  __device__ __forceinline__ void stZ(float* p, const float* v) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
  // eight input values from global memory (read-only for the whole launch)
  // u is read once (after the L2 prefetch) and y written once: both use the streaming (evict-first) cache
  // policy so they do not displace the spectrum rows that several groups of a channel share (measured 3 %
  // faster at L = 1024 and 2048, no change at longer lengths).
  // Eight input values as raw words (eight fp32 bit patterns, or four words of bf16 pairs), unpacked only
  // when the conversion reaches them, so that nothing waits on a load right after issuing it.
  __device__ __forceinline__ void ldraw(const float* p, uint32_t (&w)[8]) {
    const uint4 a = __ldcs(reinterpret_cast<const uint4*>(p)), b = __ldcs(reinterpret_cast<const uint4*>(p) + 1);
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w; w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
  }
  __device__ __forceinline__ void ldraw(const __nv_bfloat16* p, uint32_t (&w)[8]) {
    const uint4 q = __ldcs(reinterpret_cast<const uint4*>(p));
    w[0] = q.x; w[1] = q.y; w[2] = q.z; w[3] = q.w;
  }
  __device__ __forceinline__ void unpack(const float*, const uint32_t (&w)[8], float* v) {
    for (int e = 0; e < 8; e++) v[e] = __uint_as_float(w[e]);
  }
  __device__ __forceinline__ void unpack(const __nv_bfloat16*, const uint32_t (&w)[8], float* v) {
    for (int e = 0; e < 4; e++) { v[2 * e] = bf16_bits_to_float(w[e] & 0xFFFFu); v[2 * e + 1] = bf16_bits_to_float(w[e] >> 16); }
  }
  __device__ __forceinline__ void store1(float* p, float v) { __stcs(p, v); }
  __device__ __forceinline__ void store1(__nv_bfloat16* p, float v) {
    __stcs(reinterpret_cast<unsigned short*>(p), __bfloat16_as_ushort(__float2bfloat16(v)));
  }
  __device__ __forceinline__ void store4(float* p, const float* v) {
    __stcs(reinterpret_cast<float4*>(p), make_float4(v[0], v[1], v[2], v[3]));
  }
  __device__ __forceinline__ void store4(__nv_bfloat16* p, const float* v) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
    __stcs(reinterpret_cast<uint2*>(p), make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b)));
  }
  // A sequence's energy over the SEG lanes of this warp that share it (SEG lanes, aligned), stored by the
  // first of them in part[idx].
  __device__ __forceinline__ void energy_store(float* part, int idx, float ss, int seg) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1)
      if (m < seg) ss += __shfl_xor_sync(0xffffffffu, ss, m);
    if ((threadIdx.x & (seg - 1)) == 0) part[idx] = ss;
  }
  __device__ __forceinline__ void st4(uint32_t off, float v) {
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(sm + off), "f"(v));
  }
  __device__ __forceinline__ void ld4_staged(uint32_t off, uint32_t rot, float* v) {
    float w[4];
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(w[0]), "=f"(w[1]), "=f"(w[2]), "=f"(w[3]) : "r"(sm + off));
    for (int i = 0; i < 4; i++) v[i] = w[i ^ (int)rot];
  }
  // w_N^e for any integer e (reduced mod N), from the two-level table: w^(64 h) * w^l
  __device__ __forceinline__ void tw(int e, float* re, float* im) const {
    e &= (n_tw - 1);
    float hx, hy, lx, ly;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(hx), "=f"(hy) : "r"(tw_hi + (uint32_t)((e >> 6) * 8)));
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(lx), "=f"(ly) : "r"(tw_lo + (uint32_t)((e & 63) * 8)));
    *re = hx * lx - hy * ly;
    *im = hx * ly + hy * lx;
  }
  // 16 complex values (a + ib) times t0 * w^j (j < 8) and t8 * w^(j-8) (j >= 8), rounded to fp16 pairs:
  // two independent recurrences of four steps, each carrying two elements per f32x2 op.
  __device__ __forceinline__ void twiddle16(const float* a, const float* b, float t0r, float t0i, float t8r, float t8i,
                                            float wr, float wi, uint32_t* pr, uint32_t* pim) const {
    const float t1r = t0r * wr - t0i * wi, t1i = t0r * wi + t0i * wr;
    const float t9r = t8r * wr - t8i * wi, t9i = t8r * wi + t8i * wr;
    const float w2r = wr * wr - wi * wi, w2i = 2.f * wr * wi;
    u64 TR[2] = {pk2(t0r, t1r), pk2(t8r, t9r)}, TI[2] = {pk2(t0i, t1i), pk2(t8i, t9i)};
    const u64 W2R = pk2(w2r, w2r), W2I = pk2(w2i, w2i), NW2I = pk2(-w2i, -w2i), NEG = pk2(-1.f, -1.f);
#pragma unroll
    for (int q = 0; q < 4; q++) {
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int p = q + 4 * h;   // elements 2p, 2p + 1
        const u64 A = pk2(a[2 * p], a[2 * p + 1]), B = pk2(b[2 * p], b[2 * p + 1]);
        const u64 NTI = mul2(TI[h], NEG);
        const u64 ORE = fma2(B, NTI, mul2(A, TR[h]));
        const u64 OIM = fma2(A, TI[h], mul2(B, TR[h]));
        float x0, x1, z0, z1;
        up2(ORE, x0, x1);
        up2(OIM, z0, z1);
        pr[p] = pack2(x0, x1);
        pim[p] = pack2(z0, z1);
        const u64 TRn = fma2(TI[h], NW2I, mul2(TR[h], W2R));
        TI[h] = fma2(TI[h], W2R, mul2(TR[h], W2I));
        TR[h] = TRn;
      }
    }
  }
  // 16 complex values (a + ib) times the spectrum pieces kk (spec_piece format: scaled, re/im split),
  // rounded to fp16 pairs; two elements per f32x2 op.
  __device__ __forceinline__ void cmul16(const float* a, const float* b, const float* kk, uint32_t* pr,
                                         uint32_t* pim) const {
    const u64 NEG = pk2(-1.f, -1.f);
#pragma unroll
    for (int p = 0; p < 8; p++) {
      const u64 A = pk2(a[2 * p], a[2 * p + 1]), B = pk2(b[2 * p], b[2 * p + 1]);
      const u64 KR = pk2(kk[4 * p], kk[4 * p + 1]), KI = pk2(kk[4 * p + 2], kk[4 * p + 3]);
      const u64 ORE = fma2(B, mul2(KI, NEG), mul2(A, KR));
      const u64 OIM = fma2(A, KI, mul2(B, KR));
      float x0, x1, z0, z1;
      up2(ORE, x0, x1);
      up2(OIM, z0, z1);
      pr[p] = pack2(x0, x1);
      pim[p] = pack2(z0, z1);
    }
  }
};

struct BmatEmitDev {
  uint8_t* base;
  __device__ __forceinline__ void operator()(int off, int R, int q, int which, int set) {
    float s, c;
    sincospif(2.0f * (float)q / (float)R, &s, &c);
    const float v = which == 0 ? c : (which == 1 ? -s : s);
    __half h = __float2half_rn(v);
    if (set == 1) h = __float2half_rn(v - __half2float(h));   // low part of the fp16 hi+lo split
    *reinterpret_cast<__half*>(base + off) = h;
  }
};

struct ConvParams {
  const void* u;
  const float* Kf;       // [H][N] complex fp32 spectrum in digit order (float pairs)
  const uint4* btab;     // cached DFT-matrix image (BMAT_BYTES), or nullptr for in-kernel build
  void* y;
  int* status;
  int B, H;
  int ngroups;           // ceil(pairs / G), pairs = ceil(B/2) * H
  unsigned long long wait_ns;   // limit of every barrier wait, in ns (0: kWaitLimitNs)
  int debug_skip_arrive;        // test hook of sffft_debug_conv_timeout: g + 1 makes the first warp of the
                                // team converting group g skip its arrival, so that a barrier never completes
                                // and the bounded waits run out (0 in every regular launch)
  BlockArgs blk;                // composite plans' forward / inverse launches (kernel MODE 1 / 2) only
#ifdef SFFFT_TRACE
  unsigned long long* trace;   // debug builds only: [grid][kTraceRoles][kTraceLen] SM clock stamps
#endif
};

#ifdef SFFFT_TRACE
// roles: 0 L2 prefetcher, 1 MMA issuer, 2 + t compute team t (its first warp's lane 0)
constexpr int kTraceLen = 2048, kTraceRoles = 8;
#define SFFFT_STAMP(role, idx)                                                                         \
  do {                                                                                                 \
    if (prm.trace && (idx) < kTraceLen)                                                                \
      prm.trace[((size_t)blockIdx.x * kTraceRoles + (role)) * kTraceLen + (idx)] = clock64();          \
  } while (0)
#else
#define SFFFT_STAMP(role, idx) \
  do {                         \
  } while (0)
#endif

// ---- extra PTX used only by the persistent kernel ----
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Bounded wait that also gives up when another role has aborted.
__device__ __forceinline__ bool wait_phase(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_ns() - t0 > s_wait_ns) { *abort_flag = 1; return false; }
  }
}

// Every lane of the warp waits on the barrier itself (each lane then sees the data the phase publishes);
// the vote makes the outcome uniform across the warp, so warp-wide steps that follow cannot diverge.
__device__ __forceinline__ bool wait_phase_all(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const bool ok = wait_phase(bar, parity, abort_flag);
  return __all_sync(0xffffffffu, ok) != 0;
}

// A shared FIFO slot (the staged spectrum rows) is consumed by several teams out of order, so a consumer
// can reach a slot two or more uses ahead of its barrier, where a parity test cannot tell the phases
// apart.  The filler stamps each slot with the index of what it is filling before it arms the barrier; a
// consumer first waits (bounded) until the stamp reaches its own index, after which the barrier's pending
// phase is its own and the parity wait is exact.  The same bounded wait serves the prefetcher's count of
// converted groups.
__device__ __forceinline__ bool wait_stamp(const volatile int* stamp, int want, volatile int* abort_flag) {
  if (*stamp >= want) return true;
  const uint64_t t0 = global_ns();
  while (*stamp < want) {
    if (*abort_flag) return false;
    if (global_ns() - t0 > s_wait_ns) { *abort_flag = 1; return false; }
    __nanosleep(64);   // polling warps would otherwise take issue slots from the compute warps
  }
  return true;
}
__device__ __forceinline__ bool wait_stamp_all(const volatile int* stamp, int want, volatile int* abort_flag) {
  const bool ok = wait_stamp(stamp, want, abort_flag);
  return __all_sync(0xffffffffu, ok) != 0;
}

// One arrival per warp on a consumer barrier (initialised with the number of arriving warps): the warp's
// lanes finish their own accesses and fences first, the warp synchronises, then lane 0 arrives.
__device__ __forceinline__ void warp_arrive(uint64_t* bar, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
}

template <class P, bool ACC16, bool LO, int SID>
__device__ __forceinline__ void issue_sid(DevOps& ops, uint32_t tmem, uint32_t data_s, uint32_t bmat_s) {
  issue_stage<P, ACC16, SID, LO>(ops, tmem, data_s, bmat_s);
}

template <class P, bool ACC16, bool LO>
__device__ void issue_any(int sid, DevOps& ops, uint32_t tmem, uint32_t data_s, uint32_t bmat_s) {
  switch (sid) {
    case 0: issue_sid<P, ACC16, LO, 0>(ops, tmem, data_s, bmat_s); break;
    case 1: issue_sid<P, ACC16, LO, 1>(ops, tmem, data_s, bmat_s); break;
    case 2: issue_sid<P, ACC16, LO, 2>(ops, tmem, data_s, bmat_s); break;
    case 3: issue_sid<P, ACC16, LO, 3>(ops, tmem, data_s, bmat_s); break;
    default:
      if constexpr (P::S == 3) {
        if (sid == 4) issue_sid<P, ACC16, LO, 4>(ops, tmem, data_s, bmat_s);
        else issue_sid<P, ACC16, LO, 5>(ops, tmem, data_s, bmat_s);
      }
  }
}

template <class P, class TIO, bool ACC16, int SID>
__device__ __forceinline__ void epi_sid(DevOps& ops, const EpiArgs& ea, const GroupPairs& gp, int q, int wi, int lane) {
  epi_warp<P, TIO, ACC16, SID>(ops, ea, gp, wi, q, lane);
}

template <class P, class TIO, bool ACC16>
__device__ void epi_any(int sid, DevOps& ops, const EpiArgs& ea, const GroupPairs& gp, int q, int wi, int lane) {
  if constexpr (!shared_twiddle<P, TIO>()) {
    switch (sid) {
      case 0: epi_sid<P, TIO, ACC16, 0>(ops, ea, gp, q, wi, lane); break;
      case 1: epi_sid<P, TIO, ACC16, 1>(ops, ea, gp, q, wi, lane); break;
      case 2: epi_sid<P, TIO, ACC16, 2>(ops, ea, gp, q, wi, lane); break;
      case 3: epi_sid<P, TIO, ACC16, 3>(ops, ea, gp, q, wi, lane); break;
      default:
        if constexpr (P::S == 3) {
          if (sid == 4) epi_sid<P, TIO, ACC16, 4>(ops, ea, gp, q, wi, lane);
          else epi_sid<P, TIO, ACC16, 5>(ops, ea, gp, q, wi, lane);
        }
    }
  } else if (sid == 2) {
    epi_sid<P, TIO, ACC16, 2>(ops, ea, gp, q, wi, lane);
  } else if (sid == 5) {
    epi_sid<P, TIO, ACC16, 5>(ops, ea, gp, q, wi, lane);
  } else {
    // the four twiddle stages share one copy of the epilogue; the stage only selects its constants
    TwParams tp;
    switch (sid) {
      case 0: tp = tw_params<P, 0>(); break;
      case 1: tp = tw_params<P, 1>(); break;
      case 3: tp = tw_params<P, (P::S == 3 ? 3 : 0)>(); break;
      default: tp = tw_params<P, (P::S == 3 ? 4 : 0)>(); break;
    }
    twiddle_stage<P, TIO, ACC16>(ops, ea, tp, wi, q, lane);
  }
}

// Barrier over one team of compute warps, on the team's mbarrier (one arrival per warp) with the same
// bounded wait as every other wait in the kernel; `phase` is the caller's count of earlier uses.
__device__ __forceinline__ bool team_sync(uint64_t* bar, uint32_t& phase, int lane, volatile int* abort_flag) {
  warp_arrive(bar, lane);
  const bool ok = wait_phase_all(bar, phase & 1u, abort_flag);
  phase++;
  return ok;
}

// Whether any row of the group is scaled (pair_scales), the lanes of one warp in parallel: lane j < 2G sums
// row j's energy slots, gets its partner row's energy by a shuffle and derives its row's exponent.  Every
// warp of the team reads the same slots and reaches the same answer.
template <class P, int NT>
__device__ __forceinline__ bool group_rescaled_warp(const float* en, int lane) {
  using EN = Energy<P, NT>;
  constexpr int NSQ = 2 * P::G;
  static_assert(NSQ <= 32, "rows per group");
  float e = 0.f;
  if (lane < NSQ)
    for (int i = 0; i < EN::SPS; i++) e += en[lane * EN::SPS + i];
  const float ep = __shfl_xor_sync(0xffffffffu, e, 1);
  int f0 = 0, f1 = 0;
  if (lane < NSQ) {
    if (lane & 1) pair_exponents(ep, e, P::L, &f0, &f1);
    else pair_exponents(e, ep, P::L, &f0, &f1);
  }
  return __any_sync(0xffffffffu, ((lane & 1) ? f1 : f0) != 0) != 0;
}

// The second conversion pass of a group with a row to rescale (rare), out of line so that it adds nothing to
// the register allocation of the kernel's main loop.
template <class P, class TIO, int NB, int NT>
__device__ __noinline__ void convert_scaled(DevOps ops, const TIO* u, GroupPairs gp, int tid, const float* en) {
  const int j = tid / Energy<P, NT>::TPS;
  convert_group<P, TIO, NB, NT>(ops, u, gp, tid, nullptr, row_in_scale<P, NT>(en, j >> 1, j & 1));
}

// MODE 0: the convolution in one launch.  Composite plans run a partitioned convolution in two launches over
// the blocks of their rows (BlockArgs): MODE 1 converts the input blocks and runs the forward stages, storing
// the pair spectra; MODE 2 sums the spectra times the filter's block spectra and runs the inverse stages.
template <class P, class TIO, bool ACC16, int MODE = 0>
__global__ void __launch_bounds__(Shape<P, sizeof(TIO)>::NT, 1) fused_conv_kernel(ConvParams prm) {
  using SH = Shape<P, sizeof(TIO)>;
  constexpr int S2 = 2 * P::S, NS = SH::NS;
  constexpr int NSTG = MODE == 0 ? S2 : P::S;   // stages a launch runs per group
  constexpr int SID0 = MODE == 2 ? P::S : 0;    // its first stage
  constexpr int TPG = NSTG + 1;                 // tasks per group: conversion (or spectrum sums) + epilogues
  static_assert(MODE == 0 || TPG < SH::TPG, "modes");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* bmat = sm;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + SH::BAR_OFF);
  uint64_t* a_ready = bars;                    // [NS]  a team wrote a stage operand of this slot
  uint64_t* mma_done = a_ready + NS;           // [NS]  a stage's MMAs of this slot completed
  uint64_t* k_full = mma_done + NS;            // [2]   spectrum rows staged
  uint64_t* k_empty = k_full + 2;              // [2]   staged spectrum consumed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(k_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(k_empty + 3);
  int* kinfo = reinterpret_cast<int*>(k_empty + 4);   // [2] first staged channel, or -1
  uint64_t* team_done = k_empty + 5;           // [NTEAM] a team's warps staged their outputs / copied them out
  uint64_t* bmat_full = team_done + SH::NTEAM; // the cached DFT matrices have arrived (bulk copy)
  volatile int* kstamp = reinterpret_cast<volatile int*>(bmat_full + 1);   // [2] group being staged
  volatile int* conv_done = kstamp + 2;        // groups whose input has been converted
  volatile int* rep = conv_done + 1;           // [NS] the slot's next MMA request repeats stage 0
  uint8_t* kstage = sm + SH::K_OFF;
  // per slot and round parity: the group's energy slots, written by its team's conversion
  float* energies = reinterpret_cast<float*>(sm + SH::EN_OFF);   // [NS][2][EN_STRIDE]
  static_assert(Energy<P, SH::TWARPS * 32>::SLOTS == SH::EN_STRIDE, "energy area");

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ni = (int)blockIdx.x < prm.ngroups ? (prm.ngroups - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;

  // the next kernel of the stream may start its own prologue as soon as SMs free up (it waits for this grid to
  // complete before touching global memory)
  if (tid == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (warp == 1) { tmem_alloc(tmem_slot, SH::TMEM_ALLOC); tmem_relinquish(); }
  if (tid == 0) {
    // consumer barriers count one arrival per warp of the consuming team
    for (int s = 0; s < NS; s++) { mbar_init(a_ready + s, SH::TWARPS); mbar_init(mma_done + s, 1); }
    for (int l = 0; l < 2; l++) { mbar_init(k_full + l, 32); mbar_init(k_empty + l, SH::TWARPS); }
    for (int t = 0; t < SH::NTEAM; t++) mbar_init(team_done + t, SH::TWARPS);
    mbar_init(bmat_full, 1);
    kstamp[0] = kstamp[1] = -1;
    *conv_done = 0;
    for (int q = 0; q < NS; q++) rep[q] = 0;
    *abort_flag = 0;
    s_wait_ns = prm.wait_ns ? prm.wait_ns : kWaitLimitNs;
    fence_mbar_init();
    // the cached DFT matrices arrive by bulk copy while the teams convert their first groups; the MMA warp waits
    // for them before its first issue
    if (prm.btab) bulk_load_smem(bmat, prm.btab, P::BMAT_BYTES, bmat_full);
  }
  if (!prm.btab) {
    BmatEmitDev emit{bmat};
    for_each_bmat_entry<P>(emit, tid, SH::NT);
  }
  float2* tw_lo = reinterpret_cast<float2*>(sm + SH::TW_OFF);
  float2* tw_hi = tw_lo + 64;
  for (int i = tid; i < 64 + P::N / 64; i += SH::NT) {
    // exact arguments: w_N^e = exp(-2 pi i e / N) with e reduced to (-N/2, N/2]
    int e = i < 64 ? i : 64 * (i - 64);
    if (e > P::N / 2) e -= P::N;
    float sn, cs;
    sincospif(-2.0f * (float)e / (float)P::N, &sn, &cs);
    tw_lo[i] = make_float2(cs, sn);
  }
  const TIO* u = reinterpret_cast<const TIO*>(prm.u);
  // L2 prefetch of group gi's input sequences and spectrum rows by warp 0 (one bulk prefetch per sequence; the
  // inverse launch of a composite plan: each pair's summed spectrum row).  A prefetch only moves lines into L2, the
  // point of coherence, so it may be issued before the previous kernel has finished writing them: the loads that
  // use the data come after the dependency wait below.
  auto prefetch_group = [&](int gi) {
    const int group = (int)blockIdx.x + gi * (int)gridDim.x;
    const GroupPairs gp = group_pairs(group, P::G, prm.B, prm.H);
    if constexpr (MODE == 2) {
      if (lane < P::G) {
        const PairInfo pi = gp.get(lane, P::L);
        const int hb = pi.h >> prm.blk.lgP, pb = pi.h - (hb << prm.blk.lgP);
        if (pi.h >= 0)
          prefetch_l2(prm.blk.Z + 2 * ((((long long)(hb << prm.blk.lgP) + pb) * gp.PB + pi.j) * P::N), P::N * 8);
      }
      return;
    }
    if (lane < 2 * P::G) {
      const PairInfo pi = gp.get(lane >> 1, P::L);
      const long long off = (lane & 1) ? pi.off1 : pi.off0;
      if (off >= 0) prefetch_l2(u + off, (uint32_t)SH::SEQB);
    }
    if (MODE == 0 && lane == 0) {
      const PairInfo a = gp.get(0, P::L), b = gp.get(P::G - 1, P::L);
      if (a.h >= 0) prefetch_l2(prm.Kf + 2ll * a.h * P::N, P::N * 8);
      if (b.h >= 0 && b.h != a.h) prefetch_l2(prm.Kf + 2ll * b.h * P::N, P::N * 8);
    }
  };
  // the first PD groups' prefetches overlap the previous kernel's tail
  const int npre = ni < SH::PD ? ni : SH::PD;
  if (warp == 0)
    for (int gi = 0; gi < npre; gi++) prefetch_group(gi);
  // everything above touched only shared memory, TMEM and the plan's constant DFT-matrix image (and issued L2
  // prefetches); u, Kf, y and the status word may be produced or consumed by the stream's previous kernel, which
  // must have completed first
  asm volatile("griddepcontrol.wait;" ::: "memory");
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- L2 prefetcher ----------------
    // Brings each group's 2G input sequences (one bulk prefetch per sequence, one lane each) and spectrum
    // rows into L2, at most PD groups ahead of the conversions, so a team's direct loads hit L2.
    for (int gi = npre; gi < ni; gi++) {
      if (gi >= SH::PD && !wait_stamp_all(conv_done, gi - SH::PD + 1, abort_flag)) break;
      if (lane == 0) SFFFT_STAMP(0, 3 * gi);
      prefetch_group(gi);
      if (lane == 0) SFFFT_STAMP(0, 3 * gi + 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // Slot s holds this CTA's groups s, s + NS, ...; each group needs its 2S stages in order.  The issuer
    // scans the slots and issues the next stage of any slot whose operand is ready.
    if (lane == 0 && (!prm.btab || wait_phase(bmat_full, 0u, abort_flag))) {
      DevOps ops{smem_u32(sm), ACC16, 0u, 0u, P::N};
      int done[NS], total[NS], ncommit[NS];
      uint32_t ar_bits = 0;
      int left = 0;
#pragma unroll
      for (int s = 0; s < NS; s++) {
        done[s] = 0;
        ncommit[s] = 0;
        total[s] = (s < ni ? (ni - s + NS - 1) / NS : 0) * NSTG;
        left += total[s];
      }
      int nmma = 0;
      (void)nmma;
      uint64_t t_idle = global_ns();
      uint32_t idle = 0;
      while (left > 0) {
        bool progressed = false;
#pragma unroll
        for (int s = 0; s < NS; s++) {
          if (done[s] < total[s] && mbar_test_wait(a_ready + s, (ar_bits >> s) & 1u)) {
            SFFFT_STAMP(1, 3 * nmma);
            ar_bits ^= 1u << s;
            tc_fence_after();
            SFFFT_STAMP(1, 3 * nmma + 1);
            // a team that converted its group again, rescaled, asks for stage 0 once more (rep, set before its
            // arrival)
            const bool again = rep[s] != 0;
            if (again) rep[s] = 0;
            issue_any<P, ACC16, sizeof(TIO) == 4>(SID0 + (again ? done[s] - 1 : done[s]) % NSTG, ops,
                                tmem + (uint32_t)(s * P::TMEM_COLS),
                                smem_u32(sm + SH::DATA_OFF + s * P::DATA_BYTES), smem_u32(bmat));
            mma_commit(mma_done + s);
            SFFFT_STAMP(1, 3 * nmma + 2);
            nmma++;
            ncommit[s]++;
            if (!again) {
              done[s]++;
              left--;
            }
            progressed = true;
          }
        }
        if (progressed) {
          t_idle = global_ns();
          idle = 0;
        } else if ((++idle & 15u) == 0) {
          // the abort flag and the time limit are checked every 16th idle scan, so a scan is only the slots'
          // barrier tests
          if (*abort_flag) break;
          if (global_ns() - t_idle > s_wait_ns) { *abort_flag = 1; break; }
          // nothing ready: poll again at once (sleeping 32 or 128 ns between polls measured 0.5-1 % slower; the
          // issue slots the spin takes from the compute warps on this scheduler cost less than the delay)
        }
      }
      // make sure no MMA is still writing TMEM when the CTA frees it
#pragma unroll
      for (int s = 0; s < NS; s++) {
        if (!ncommit[s]) continue;
        const uint64_t t0 = global_ns();
        while (!mbar_try_wait(mma_done + s, (uint32_t)((ncommit[s] - 1) & 1)) && global_ns() - t0 < s_wait_ns) {
        }
      }
    }
  } else if (warp == 2) {
    // ---------------- spectrum loader ----------------
    // Copies each group's spectrum rows (coalesced 16-byte loads) into a staging slot in the swizzled
    // order the spectrum epilogue reads; a group whose pairs span more than KC channels is marked -1 and
    // its epilogue reads Kf from global memory instead.
    if constexpr (SH::KSLOT > 0 && MODE == 0) {
      constexpr int NPIECE = SH::KROW / 16, PPR = P::RL / 2;   // 16-byte pieces per row of the last digit
      for (int gi = 0; gi < ni; gi++) {
        const int ks = gi % SH::KSLOT, use = gi / SH::KSLOT;
        if (use > 0) {
          if (!wait_phase_all(k_empty + ks, (uint32_t)((use - 1) & 1), abort_flag)) break;
        }
        if (lane == 0) kstamp[ks] = gi;
        const int group = (int)blockIdx.x + gi * (int)gridDim.x;
        const GroupPairs gp = group_pairs(group, P::G, prm.B, prm.H);
        const int hf = gp.get(0, P::L).h;
        int hl = hf;
        for (int g = P::G - 1; g > 0; g--) {
          const int h = gp.get(g, P::L).h;
          if (h >= 0) { hl = h; break; }
        }
        const bool staged = hf >= 0 && hl - hf + 1 <= SH::KC;
        if (staged) {
          uint8_t* kb = kstage + ks * SH::KC * SH::KROW;
          for (int ci = 0; ci <= hl - hf; ci++) {
            const uint4* src = reinterpret_cast<const uint4*>(prm.Kf + 2ll * (hf + ci) * P::N);
            uint8_t* dst = kb + ci * SH::KROW;
            for (int o0 = 0; o0 < NPIECE; o0 += 256) {
              uint4 v[8];
#pragma unroll
              for (int q2 = 0; q2 < 8; q2++) {
                const int o = o0 + q2 * 32 + lane;
                v[q2] = o < NPIECE ? __ldg(src + o) : make_uint4(0, 0, 0, 0);
              }
#pragma unroll
              for (int q2 = 0; q2 < 8; q2++) {
                const int o = o0 + q2 * 32 + lane;
                if (o < NPIECE) {
                  const int rr = o / PPR, rem = o - rr * PPR;
                  float raw[4] = {__uint_as_float(v[q2].x), __uint_as_float(v[q2].y), __uint_as_float(v[q2].z),
                                  __uint_as_float(v[q2].w)};
                  float pc[4];
                  spec_piece(raw, stage_scale(P::RL), pc);
                  *reinterpret_cast<float4*>(dst + kstage_off<P::N, P::RL>(rr, rem >> 3, rem & 7)) =
                      make_float4(pc[0], pc[1], pc[2], pc[3]);
                }
              }
            }
          }
        }
        if (lane == 0) kinfo[ks] = staged ? hf : -1;
        __syncwarp();
        mbar_arrive(k_full + ks);
      }
    }
  } else {
    // ---------------- compute warps ----------------
    // Team `team` (warps team*TWARPS .. of the compute warps) owns slots team*NST .. team*NST + NST - 1
    // and, round after round, runs the TPG tasks of its groups, alternating between its slots.
    constexpr int NST = SH::NST, TWT = SH::TWARPS * 32;
    const int wc = warp - SH::CW0, team = wc / SH::TWARPS, wt = wc - team * SH::TWARPS;
    const int q = warp & 3, wi = wt >> 2, ttid = wt * 32 + lane;
    uint32_t md_bits = 0;                 // bit l: parity of local slot l's next mma_done phase
    uint32_t ts_phase = 0;                // uses of this team's team_done barrier
    GroupPairs gps[NST];
    const int rounds = (ni + NS - 1) / NS;
    bool ok = true;
    int ntask = 0;
    (void)ntask;
    for (int k = 0; k < rounds * TPG && ok; k++) {
      const int j = k % TPG;
#pragma unroll
      for (int l = 0; l < NST; l++) {
        if (!ok) break;
        const int s = team * NST + l;
        const int gi = NS * (k / TPG) + s;
        if (gi >= ni) continue;
        const int group = (int)blockIdx.x + gi * (int)gridDim.x;
        if (j == 0) gps[l] = group_pairs(group, P::G, prm.B, prm.H);
        const GroupPairs gp = gps[l];
        DevOps ops{smem_u32(sm + SH::DATA_OFF + s * P::DATA_BYTES), ACC16, smem_u32(tw_lo), smem_u32(tw_hi), P::N};
        if (lane == 0 && wt == 0) SFFFT_STAMP(2 + team, 3 * ntask);
        if (j == 0) {
          // convert the group's input, measuring each row's energy for the MMA warp, which derives the rows'
          // scales while the stage-0 MMAs run (pair_scales)
          float* en = energies + (s * 2 + ((gi / NS) & 1)) * SH::EN_STRIDE;
          if constexpr (MODE == 0) {
            convert_group<P, TIO, SH::NB, TWT>(ops, u, gp, ttid, en, 1.f);
          } else {
            // composite: the rows' scales follow from their energies over the whole row (every warp writes
            // the same values into the slots it then reads)
            fill_energies<P, TWT>(en, prm.blk, gp, lane, 32);
            __syncwarp();
            if constexpr (MODE == 1) {
              convert_scaled<P, TIO, SH::NB, TWT>(ops, u, gp, ttid, en);
            } else {
              spec_load_units<P, TIO>(ops, prm.blk, gp, wi, q, lane);
            }
          }
          if (lane == 0 && wt == 0) SFFFT_STAMP(2 + team, 3 * ntask + 1);
          fence_async_smem();
          tc_fence_before();
          if (!(prm.debug_skip_arrive == group + 1 && wt == 0)) warp_arrive(a_ready + s, lane);
          if (lane == 0 && wt == 0) atomicAdd((int*)conv_done, 1);
          if (lane == 0 && wt == 0) SFFFT_STAMP(2 + team, 3 * ntask + 2);
        } else {
          const int sid = SID0 + j - 1;
          if (!wait_phase_all(mma_done + s, (md_bits >> l) & 1u, abort_flag)) { ok = false; break; }
          md_bits ^= 1u << l;
          // stage 0 ran after every warp of the team had converted the group (each arrived on a_ready after
          // storing its energy slots), so every warp now derives the same row scales into its own copy; a group
          // with a row to rescale (rare) is converted again with them and stage 0 repeated
          float* en = energies + (s * 2 + ((gi / NS) & 1)) * SH::EN_STRIDE;
          if (MODE == 0 && sid == 0 && group_rescaled_warp<P, TWT>(en, lane)) {
            tc_fence_after();
            convert_scaled<P, TIO, SH::NB, TWT>(ops, u, gp, ttid, en);
            if (lane == 0 && wt == 0) rep[s] = 1;
            fence_async_smem();
            tc_fence_before();
            warp_arrive(a_ready + s, lane);
            if (!wait_phase_all(mma_done + s, (md_bits >> l) & 1u, abort_flag)) { ok = false; break; }
            md_bits ^= 1u << l;
          }
          if (lane == 0 && wt == 0) SFFFT_STAMP(2 + team, 3 * ntask + 1);
          tc_fence_after();
          EpiArgs ea{tmem + (uint32_t)(s * P::TMEM_COLS), prm.Kf, prm.y, prm.B, prm.H, group, nullptr, 0, en};
          const bool kst = MODE == 0 && SH::KSLOT > 0 && sid == P::S - 1;
          constexpr int KS = SH::KSLOT > 0 ? SH::KSLOT : 1;
          const int ks = gi % KS;
          if (kst) {
            if (!wait_stamp_all(kstamp + ks, gi, abort_flag) ||
                !wait_phase_all(k_full + ks, (uint32_t)((gi / KS) & 1), abort_flag)) {
              ok = false;
              break;
            }
            const int hf = kinfo[ks];
            if (hf >= 0) { ea.kst = kstage + ks * SH::KC * SH::KROW; ea.khf = hf; }
          }
          if (MODE == 1 && sid == P::S - 1) spec_store_units<P, TIO>(ops, ea, prm.blk, gp, wi, q, lane);
          else epi_any<P, TIO, ACC16>(sid, ops, ea, gp, q, wi, lane);
          if (kst) warp_arrive(k_empty + ks, lane);
          tc_fence_before();
          if (P::S == 3 && sid == S2 - 1) {
            // 3-stage plans stage the outputs in shared memory; the team then copies them out coalesced
            if (!team_sync(team_done + team, ts_phase, lane, abort_flag)) { ok = false; break; }
            copy_out_staged<P, TIO>(ops, ea, gp, ttid, TWT);
            if (!team_sync(team_done + team, ts_phase, lane, abort_flag)) { ok = false; break; }
          }
          if (j < TPG - 1) {
            fence_async_smem();
            warp_arrive(a_ready + s, lane);
          }
          if (lane == 0 && wt == 0) SFFFT_STAMP(2 + team, 3 * ntask + 2);
        }
        ntask++;
      }
    }
  }

  // no bulk copy may still be writing shared memory when the CTA exits (it lands within microseconds; the MMA
  // warp normally waited for it long before)
  if (tid == 0 && prm.btab) mbar_wait_bounded(bmat_full, 0u, s_wait_ns);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // after the block barrier every role has finished, so an abort raised by any of them is seen here
  if (tid == 0 && *abort_flag) atomicExch(prm.status, SFFFT_ERR_TIMEOUT);
  if (warp == 1) tmem_dealloc(tmem, SH::TMEM_ALLOC);
}

}  // namespace sffft
