// Plan catalog: X(R0, R1, R2, G, W, "name/wW").
//
// The (plan, warps) pairs for L = 128..8192 are the 28 candidates the reference sweeps
// (sfFFT src/sffft.cu:506-513), so calibration output keeps its row count.  G (pairs of
// sequences per CTA) is the B200 choice: the smallest power of two that gives every stage a whole
// number of 128-row tcgen05 tiles (G * N / R_j divisible by 128).  L = 16384 (N = 32768) is new:
// 128 KiB of fp16 data plus 20 KiB of split DFT matrices fits B200's 227 KiB per-block shared memory.
#pragma once

#include "calibration.h"

#define SFFFT_CATALOG(X)                                                                              \
  X(16, 16, 1, 8, 4, "16x16/w4") X(16, 16, 1, 8, 8, "16x16/w8")                                       \
  X(32, 16, 1, 8, 4, "32x16/w4") X(16, 32, 1, 8, 4, "16x32/w4") X(32, 16, 1, 8, 8, "32x16/w8")        \
  X(32, 32, 1, 4, 4, "32x32/w4") X(32, 32, 1, 4, 8, "32x32/w8") X(64, 16, 1, 8, 4, "64x16/w4")        \
  X(16, 64, 1, 8, 4, "16x64/w4")                                                                      \
  X(64, 32, 1, 4, 4, "64x32/w4") X(32, 64, 1, 4, 4, "32x64/w4") X(64, 32, 1, 4, 8, "64x32/w8")        \
  X(32, 64, 1, 4, 8, "32x64/w8")                                                                      \
  X(16, 16, 16, 1, 4, "16x16x16/w4") X(16, 16, 16, 1, 8, "16x16x16/w8") X(64, 64, 1, 2, 8, "64x64/w8")\
  X(64, 64, 1, 2, 4, "64x64/w4")                                                                      \
  X(32, 16, 16, 1, 4, "32x16x16/w4") X(16, 32, 16, 1, 4, "16x32x16/w4")                               \
  X(16, 16, 32, 1, 4, "16x16x32/w4") X(32, 16, 16, 1, 8, "32x16x16/w8")                               \
  X(16, 16, 32, 1, 8, "16x16x32/w8")                                                                  \
  X(32, 32, 16, 1, 4, "32x32x16/w4") X(16, 32, 32, 1, 4, "16x32x32/w4") X(64, 16, 16, 1, 4, "64x16x16/w4") \
  X(32, 32, 16, 1, 8, "32x32x16/w8") X(16, 32, 32, 1, 8, "16x32x32/w8") X(16, 16, 64, 1, 8, "16x16x64/w8") \
  X(32, 32, 32, 1, 4, "32x32x32/w4") X(32, 32, 32, 1, 8, "32x32x32/w8")

// The plans with small-launch variants: the calibrated default plan of each length up to 8192 (calibration.h; the
// 16384 plan already has one slot).
constexpr bool small_variants(int R0, int R1, int R2, int W) {
  return calibrated_default(R0, R1, R2, W) && R0 * R1 * R2 <= 16384;
}

// The block plans of composite plans with the partitioned-convolution kernels: the calibrated default of every
// length (32x32x32/w8, the 16384 default, is the block of every default composite length) and 16x16/w4.
constexpr bool block_mode_plans(int R0, int R1, int R2, int W) {
  return calibrated_default(R0, R1, R2, W) || (R0 == 16 && R1 == 16 && R2 == 1 && W == 4);
}
