// Bit-exact single-precision exp shared by the host (table generator, tests)
// and the device kernels.
//
// The reference's softmax and SiLU call std::exp(float), i.e. the host libm's
// expf (reference src/ops_cpu.cpp:334 and :424), which is not correctly
// rounded. A device kernel reproduces it in two parts:
//   1. mi_expf_core(): an exp evaluated in double precision and rounded once
//      to float. Method: Tang's table-driven reduction x = (64m + j) ln2/64 + r
//      with |r| <= ln2/128, exp(r) - 1 by its degree-6 Taylor polynomial
//      (truncation < 2^-64), times 2^(j/64) from a 64-entry table and 2^m.
//      Every constant is derived from ln 2, 1/k! and 2^(j/64) (written out by
//      exp_constants.py); the code uses only +, *, fma and bit moves, so the
//      host build (gcc -ffp-contract=off) and the device build (nvcc
//      -fmad=false) produce the same bits for every input.
//   2. An exception table: every float x for which the host libm's expf(x)
//      differs from mi_expf_core(x), found by running both over all 2^32
//      inputs (mi_expf_gen), stored as a two-choice bucketed hash so one
//      device lookup costs one round of independent 16-byte loads.
#pragma once

#include <stdint.h>
#include <string.h>

#include <math.h>

#ifdef __CUDACC__
#define MI_HD __host__ __device__ __forceinline__
#else
#define MI_HD static inline
#endif

#if defined(__CUDA_ARCH__)
#define MI_FMA(a, b, c) __fma_rn((a), (b), (c))
#define MI_MUL(a, b) __dmul_rn((a), (b))
#define MI_ADD(a, b) __dadd_rn((a), (b))
#define MI_SUB(a, b) __dsub_rn((a), (b))
#else
#define MI_FMA(a, b, c) fma((a), (b), (c))
#define MI_MUL(a, b) ((a) * (b))
#define MI_ADD(a, b) ((a) + (b))
#define MI_SUB(a, b) ((a) - (b))
#endif

#include "mi_exp2_table.h"  // MI_EXP2_TAB_INIT: 2^(j/64), correctly rounded

#ifdef __CUDACC__
static __device__ const double mi_exp2_tab_dev[64] = MI_EXP2_TAB_INIT;
#endif
static const double mi_exp2_tab_host[64] = MI_EXP2_TAB_INIT;

MI_HD double mi_exp2_tab(int j) {
#ifdef __CUDA_ARCH__
  return mi_exp2_tab_dev[j];
#else
  return mi_exp2_tab_host[j];
#endif
}

MI_HD double mi_asdouble(uint64_t u) {
#ifdef __CUDA_ARCH__
  return __longlong_as_double((long long)u);
#else
  double d;
  memcpy(&d, &u, 8);
  return d;
#endif
}

MI_HD uint64_t mi_asuint64(double d) {
#ifdef __CUDA_ARCH__
  return (uint64_t)__double_as_longlong(d);
#else
  uint64_t u;
  memcpy(&u, &d, 8);
  return u;
#endif
}

MI_HD uint32_t mi_f2u(float f) {
#ifdef __CUDA_ARCH__
  return (uint32_t)__float_as_uint(f);
#else
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
#endif
}

MI_HD float mi_u2f(uint32_t u) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float f;
  memcpy(&f, &u, 4);
  return f;
#endif
}

// exp(x) in double, before the final rounding; for -110 <= x <= 100.
MI_HD double mi_expf_core_wide(float x) {
  const double inv_ln2_64 = 0x1.71547652b82fep+6;  // 64 / ln 2
  const double shift = 0x1.8p52;                    // round-to-int by addition
  const double ln2_64_hi = 0x1.62e42fefa39efp-7;    // ln 2 / 64, leading part
  const double ln2_64_lo = 0x1.abc9e3b39803fp-62;   // ln 2 / 64, trailing part
  double xd = (double)x;
  double t = MI_ADD(MI_MUL(xd, inv_ln2_64), shift);
  double kd = MI_SUB(t, shift);
  int64_t k = (int64_t)kd;
  double r = MI_FMA(-kd, ln2_64_hi, xd);
  r = MI_FMA(-kd, ln2_64_lo, r);
  double p = 0x1.6c16c16c16c17p-10;        // 1/720
  p = MI_FMA(p, r, 0x1.1111111111111p-7);  // 1/120
  p = MI_FMA(p, r, 0x1.5555555555555p-5);  // 1/24
  p = MI_FMA(p, r, 0x1.5555555555555p-3);  // 1/6
  p = MI_FMA(p, r, 0x1.0000000000000p-1);  // 1/2
  p = MI_FMA(p, r, 1.0);
  p = MI_MUL(p, r);                        // exp(r) - 1
  int j = (int)(k & 63);
  int64_t m = k >> 6;
  double tj = mi_exp2_tab(j);
  double y = MI_FMA(tj, p, tj);
  double s = mi_asdouble((uint64_t)(1023 + m) << 52);
  return MI_MUL(y, s);
}

// exp(x) in double, rounded once to float. NaN propagates; results beyond the
// float range saturate to inf / 0 the way the final conversion rounds them.
MI_HD float mi_expf_core(float x) {
  if (!(x == x)) return x;
  if (x > 100.0f) return mi_u2f(0x7f800000u);
  if (x < -110.0f) return 0.0f;
  return (float)mi_expf_core_wide(x);
}

// Whether the double value yd lies within `thresh_bits` / 2^29 of a float
// spacing from a rounding boundary of the float grid (always true for results
// below the normal range or at the top of it). For a normal float result the
// 29 mantissa bits of yd below float precision place it within the spacing;
// the boundary is at 2^28. A libm expf whose error stays within 0.5 + eps ulp
// can only round differently from the correctly rounded result where the exact
// value lies within about eps ulp of a boundary, so the exception table needs
// probing only near one; mi_expf_gen checks that every exception it finds is
// within MI_EXPF_TIE_VERIFIED of a boundary before it marks the table for that
// shortcut, and the device probes within the wider MI_EXPF_TIE_PROBE.
#define MI_EXPF_TIE_PROBE (1u << 23)     // 2^-6 of the spacing
#define MI_EXPF_TIE_VERIFIED (1u << 22)  // 2^-7 of the spacing
MI_HD int mi_expf_near_tie(double yd, uint32_t thresh_bits) {
  if (!(yd >= 0x1p-126 && yd < 0x1.fffffep127)) return 1;
  uint64_t u;
#ifdef __CUDA_ARCH__
  u = (uint64_t)__double_as_longlong(yd);
#else
  memcpy(&u, &yd, 8);
#endif
  const int32_t low = (int32_t)((uint32_t)u & 0x1fffffffu) - (int32_t)0x10000000;
  return (uint32_t)(low < 0 ? -low : low) < thresh_bits;
}

// Exception-table file / device layout: header, then n_buckets buckets of
// MI_EXPF_SLOTS (key, value) pairs. key = input float bits, value = libm
// result bits, empty slot key = MI_EXPF_EMPTY (a NaN pattern; NaN inputs never
// reach the lookup).
#define MI_EXPF_MAGIC 0x4658454du  // "MEXF"
#define MI_EXPF_SLOTS 4
#define MI_EXPF_EMPTY 0xffffffffu
#define MI_EXPF_FLAG_TIE_FILTER 1u

typedef struct {
  uint32_t magic;
  uint32_t log2_buckets;
  uint32_t mul1, mul2;     // odd multipliers of the two bucket hashes
  uint32_t n_entries;
  uint32_t core_checksum;  // fingerprint of mi_expf_core over a fixed sample
  uint32_t libm_checksum;  // fingerprint of the host expf over the same sample
  uint32_t flags;          // MI_EXPF_FLAG_TIE_FILTER: every exception is near a boundary (mi_expf_near_tie)
} mi_expf_table_header;

MI_HD uint32_t mi_expf_bucket(uint32_t key, uint32_t mul, uint32_t log2_buckets) {
  uint32_t h = key * mul;
  h ^= h >> 15;
  h *= 0x2c1b3c6du;
  return h >> (32 - log2_buckets);
}
