// exp(d) in double for the float differences d = y - m_y <= 0 of the exact
// tail sums, by Tang's table-driven method (P. T. P. Tang, "Table-driven
// implementation of the exponential function in IEEE floating-point
// arithmetic", ACM TOMS 15(2), 1989): d = (64 i + j) ln2/64 + r with
// |r| <= ln2/128 (+ the rounding of d 64/ln2), exp(d) = 2^i 2^(j/64) (1 + p(r)),
// p the degree-5 Taylor polynomial of exp(r) - 1 (truncation below 2^-54.6).
// With the table rounded to nearest, one rounding in the reduction and one in
// the final fma, the relative error is below 2^-51 (tests/test_exp_tail.py
// checks it against long-double expl on the host). d <= -700 gives 0 (below
// 2^-1000). Constants from gen_exp_table.py; usable in host code for tests.
#pragma once
#include <stdint.h>
#include <string.h>
#include <math.h>

#ifdef __CUDACC__
#define C4S_HD __host__ __device__ __forceinline__
#else
#define C4S_HD inline
#endif

// 2^(j/64), j = 0..63, nearest doubles
#define C4S_EXP2_J64_TABLE { \
  0x1.0000000000000p+0, 0x1.02c9a3e778061p+0, 0x1.059b0d3158574p+0, 0x1.0874518759bc8p+0, \
  0x1.0b5586cf9890fp+0, 0x1.0e3ec32d3d1a2p+0, 0x1.11301d0125b51p+0, 0x1.1429aaea92de0p+0, \
  0x1.172b83c7d517bp+0, 0x1.1a35beb6fcb75p+0, 0x1.1d4873168b9aap+0, 0x1.2063b88628cd6p+0, \
  0x1.2387a6e756238p+0, 0x1.26b4565e27cddp+0, 0x1.29e9df51fdee1p+0, 0x1.2d285a6e4030bp+0, \
  0x1.306fe0a31b715p+0, 0x1.33c08b26416ffp+0, 0x1.371a7373aa9cbp+0, 0x1.3a7db34e59ff7p+0, \
  0x1.3dea64c123422p+0, 0x1.4160a21f72e2ap+0, 0x1.44e086061892dp+0, 0x1.486a2b5c13cd0p+0, \
  0x1.4bfdad5362a27p+0, 0x1.4f9b2769d2ca7p+0, 0x1.5342b569d4f82p+0, 0x1.56f4736b527dap+0, \
  0x1.5ab07dd485429p+0, 0x1.5e76f15ad2148p+0, 0x1.6247eb03a5585p+0, 0x1.6623882552225p+0, \
  0x1.6a09e667f3bcdp+0, 0x1.6dfb23c651a2fp+0, 0x1.71f75e8ec5f74p+0, 0x1.75feb564267c9p+0, \
  0x1.7a11473eb0187p+0, 0x1.7e2f336cf4e62p+0, 0x1.82589994cce13p+0, 0x1.868d99b4492edp+0, \
  0x1.8ace5422aa0dbp+0, 0x1.8f1ae99157736p+0, 0x1.93737b0cdc5e5p+0, 0x1.97d829fde4e50p+0, \
  0x1.9c49182a3f090p+0, 0x1.a0c667b5de565p+0, 0x1.a5503b23e255dp+0, 0x1.a9e6b5579fdbfp+0, \
  0x1.ae89f995ad3adp+0, 0x1.b33a2b84f15fbp+0, 0x1.b7f76f2fb5e47p+0, 0x1.bcc1e904bc1d2p+0, \
  0x1.c199bdd85529cp+0, 0x1.c67f12e57d14bp+0, 0x1.cb720dcef9069p+0, 0x1.d072d4a07897cp+0, \
  0x1.d5818dcfba487p+0, 0x1.da9e603db3285p+0, 0x1.dfc97337b9b5fp+0, 0x1.e502ee78b3ff6p+0, \
  0x1.ea4afa2a490dap+0, 0x1.efa1bee615a27p+0, 0x1.f50765b6e4540p+0, 0x1.fa7c1819e90d8p+0, \
}

namespace c4s {

constexpr double EXP_INV_LN2_64 = 0x1.71547652b82fep+6;   // 64 / ln 2
constexpr double EXP_LN2_64_HI = 0x1.62e42fefa39efp-7;    // ln 2 / 64, leading part
constexpr double EXP_LN2_64_LO = 0x1.abc9e3b39803fp-62;    // ln 2 / 64 - EXP_LN2_64_HI

// 2^i for -1022 <= i <= 1023.
C4S_HD double exp_pow2i(int i) {
  const uint64_t b = (uint64_t)(i + 1023) << 52;
#ifdef __CUDA_ARCH__
  return __longlong_as_double((long long)b);
#else
  double r;
  memcpy(&r, &b, sizeof r);
  return r;
#endif
}

// exp(d) for d <= 0; tab = the 2^(j/64) table (C4S_EXP2_J64_TABLE).
C4S_HD double exp_tail(float d, const double* tab) {
  if (!(d > -700.0f)) return 0.0;
  const double x = (double)d;
  const double n = rint(x * EXP_INV_LN2_64);
  const int ni = (int)n;
  double r = fma(-n, EXP_LN2_64_HI, x);
  r = fma(-n, EXP_LN2_64_LO, r);
  const double p = r * (1.0 + r * (0.5 + r * (1.0 / 6.0 + r * (1.0 / 24.0 + r * (1.0 / 120.0)))));
  const double t = tab[ni & 63];
  return fma(t, p, t) * exp_pow2i(ni >> 6);
}

}  // namespace c4s
