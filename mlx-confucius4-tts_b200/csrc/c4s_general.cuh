// c4s_general.cuh -- the general (exact, any-input) path of the T2S sampling
// kernels: shared row staging and penalty, and the per-row processors that
// hold the row in shared memory. Used on its own for c4s_process / c4s_argmax
// and rows wider than the fast kernel's register capacity, and by the fast
// kernel for the rare rows it defers.
#pragma once

#include <cuda_runtime.h>

#include "../../include/c4s_sampling.h"
#include "c4s_device.cuh"

namespace c4s {

enum { MODE_SAMPLE = 0, MODE_PROCESS = 1, MODE_ARGMAX = 2 };

struct RowJob;                  // fast path: per-row job record (c4s_fast.cuh)

struct Args {
  const float* logits;          // MODE_SAMPLE / MODE_ARGMAX input
  float* inout;                 // MODE_PROCESS rows (in place)
  int B, V;
  long long ld;
  const int* hist;
  const long long* hist_off;   // CSR [B+1], or with hist_len the window starts [B]
  const int* hist_len;          // null (CSR), or per-row window lengths [B]
  long long hist_total;
  const c4s_row_params* params;
  int params_stride;
  unsigned long long* rng;
  const unsigned char* active;
  int* out_ids;
  float* out_logits;
  long long out_ld;
  int mode, stages, debug;
  double qscale;                // 2^F, fixed-point scale for probabilities
  unsigned long long* scratch;  // per-CTA sort slab for the exact top-p fallback
  int scratch_stride;           // keys per CTA (power of two >= V)
  unsigned* errflags;
  unsigned long long* counters;
  // fast path: per-row jobs and candidate lists of the current chunk, rows for the general path
  RowJob* jobs;
  unsigned long long* lkeys;    // [B][LCAP] candidate keys
  unsigned long long* lsb;      // [B][LCAP] sort buffer of the exact fallback
  int* defer_rows;              // rows handed to the general path
  int* big_rows;                // rows whose lists the list kernel works with a whole CTA
  unsigned* defer_cnt;          // [0] count, [1] CTAs of the general-path kernel done, [2] row counter,
                                // list queues: [3 + 2q]/[4 + 2q] rows queued/taken in class q
                                // (rows in big_rows + q * chunk; q = 0: long lists),
                                // [ORD_CNT + c]: rows of the row kernel's cost class c
  int* order;                   // [ROW_CLASSES][chunk] rows by cost class, dearest class first
                                // (null: the row kernel takes rows in index order)
  int chunk;                    // rows per split-path launch sequence (the stride of the queues above)
};

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct Layout {
  size_t row, bitmap, cnt, mass, key, pv, total;
};
__host__ __device__ inline Layout layout_for(int V) {
  Layout L;
  size_t o = 0;
  L.row = o;    o += align_up((size_t)(V + 4) * 4, 16);
  L.bitmap = o; o += align_up((size_t)((V + 31) / 32) * 4, 16);
  L.cnt = o;    o += NBIN * 4;
  L.mass = o;   o += NBIN * 8;
  L.key = o;    o += LIST_CAP * 8;
  L.pv = o;     o += LIST_CAP * 8;
  L.total = o;
  return L;
}

struct Shared {
  unsigned long long bar;
  unsigned long long red64[NWARP];
  float redf[NWARP];
  int redi[NWARP];
  unsigned redu[NWARP];
  unsigned long long u64a, u64b, u64c, kp, kkeep;
  double dsum;
  int c, slot, slot2, jstar, tok, abort_row, ns, nk, defer, last, done;
  unsigned cbefore, thresh_key;
  unsigned long long mbefore;
  double redd[NWARP];
  double d1, d2;
  // fast kernel (row warps)
  int dq[8];                    // rows the list warps handed back, not yet reprocessed
  int ndq;
  int abort_all;                // a bounded wait gave up: stop after this row
  double oct[32];               // octave masses of the estimate
  int nrow[2];                  // row kernel: the next row of this CTA (by iteration parity)
  float fbefore;                // mass of the sub-bins below the crossing one
};

// u = 2^-53: unit roundoff of double.
constexpr double U53 = 1.1102230246251565e-16;

// Error band (in fixed-point units) between the fixed-point prefix sums of
// n probabilities and the reference's sequentially rounded double sums,
// doubled for margin: rounding of n adds and n divisions (<= 4n+16 ulps of the
// total), exp() differences of <= 2 ulps per term, and the fixed-point
// rounding of <= 1/2 unit per term on each of the prefix and the total.
__device__ __forceinline__ double band_q(int n, double SQ) {
  return 2.0 * ((4.0 * n + 16.0) * U53 * SQ + (double)n + 2.0);
}

// IEEE division, not inlined (keeps the many call sites small).
__device__ __noinline__ float div_call(float x, float d) { return __fdiv_rn(x, d); }

// Correctly rounded x / d with rd = RN(1/d) given (one __frcp_rn per row):
// two Newton corrections of x*rd with fused remainders (Markstein, "Computation
// of elementary functions on the IBM RISC System/6000 processor", IBM J. Res.
// Dev. 34(1), 1990), then a proof check: the remainder r = x - q*d of the final
// q is exact (FMA), and |r| < |d| * ulp(q)/2 (with a 2^-20 margin) shows that q
// is the float nearest to x/d. Quotients it cannot prove -- near-ties, powers
// of two (whose lower neighbour is half an ulp away), |q| outside
// [2^-100, 2^100], d outside [2^-100, 2^100] -- come from __fdiv_rn.
//
// div_rn_try is the same without the fallback: the quotient and whether the
// proof holds. Its callers compute many quotients with no call in between
// (a possible call at every quotient keeps the compiler from overlapping
// them) and send the rare unproven ones to div_call afterwards.
__device__ __forceinline__ float div_rn_try(float x, float d, float rd, bool& ok) {
  const float q0 = __fmul_rn(x, rd);
  float r = __fmaf_rn(-q0, d, x);
  float q = __fmaf_rn(r, rd, q0);
  r = __fmaf_rn(-q, d, x);
  q = __fmaf_rn(r, rd, q);
  r = __fmaf_rn(-q, d, x);
  const unsigned bq = __float_as_uint(q) & 0x7fffffffu;
  const float hulp = __uint_as_float((bq & 0x7f800000u) - (24u << 23));   // ulp(q) / 2
  const float ad = fabsf(d);
  const bool zero = x == 0.0f;                      // signed zero (the corrections would lose -0)
  ok = zero || (bq >= 0x0d800000u && bq <= 0x71800000u && (bq & 0x007fffffu) != 0u && ad >= 7.8886e-31f &&
                ad <= 1.2676e30f && fabsf(r) < __fmul_rn(__fmul_rn(hulp, ad), 0.99999905f));
  return zero ? q0 : q;
}
__device__ __forceinline__ float div_rn(float x, float d, float rd) {
  bool ok;
  const float q = div_rn_try(x, d, rd, ok);
  return ok ? q : div_call(x, d);
}

// Not inlined: CUDA's exp(double) is large and is called from many sites.
__device__ __noinline__ double prob(float y, float m) {
  return exp((double)__fsub_rn(y, m));
}

__device__ __forceinline__ unsigned long long qfix(double p, double qscale) {
  return __double2ull_rn(__dmul_rn(p, qscale));
}

// ------------------------------------------------------------------------
// k-th largest value by 4-pass MSD radix select over fkey (general path).
// ------------------------------------------------------------------------
__device__ float radix_kth_largest(const float* srow, int V, int k, unsigned* cnt, Shared& S) {
  unsigned prefix = 0, pmask = 0, kk = (unsigned)k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int j = threadIdx.x; j < NBIN; j += NT) cnt[j] = 0;
    csync();
    for (int i = threadIdx.x; i < V; i += NT) {
      const unsigned u = fkey(srow[i]);
      if ((u & pmask) == prefix) atomicAdd(&cnt[(u >> shift) & 255u], 1u);
    }
    csync();
    if (threadIdx.x < 32)
      warp_find_bin<unsigned>([&](int j) { return cnt[255 - j]; }, kk, false, &S.c, &S.cbefore);
    csync();
    const unsigned d = 255u - (unsigned)S.c;
    kk -= S.cbefore;
    prefix |= d << shift;
    pmask |= 0xffu << shift;
    csync();
  }
  return fkey_inv(prefix);
}

// Gather keys ckey(y,i) of all elements with pred(y, i) into lkey[0..n), pad to
// a power of two and sort ascending. Returns n (caller guarantees n <= LIST_CAP).
template <typename Pred>
__device__ int gather_sort(const float* srow, int V, unsigned long long* lkey, Shared& S, Pred pred,
                           bool index_keys) {
  if (threadIdx.x == 0) S.slot = 0;
  csync();
  for (int i = threadIdx.x; i < V; i += NT) {
    const float y = srow[i];
    if (pred(y, i)) {
      const int s = atomicAdd(&S.slot, 1);
      if (s < LIST_CAP) lkey[s] = index_keys ? (unsigned long long)i : ckey(y, i);
    }
  }
  csync();
  const int n = min(S.slot, LIST_CAP);
  const int np = next_pow2(max(n, 1));
  for (int p = n + threadIdx.x; p < np; p += NT) lkey[p] = KEY_MAX;
  csync();
  bitonic_sort_u64(lkey, np);
  return n;
}

// Exact reference top-p sums over keys K[0..n) sorted ascending, sequentially
// by one thread; returns the first position whose cumulative probability is
// above 1-p (n if none). pv is scratch of >= NT doubles; K may be global.
__device__ int topp_exact_seq(const float* srow, const unsigned long long* K, int n, float m, float p,
                              double* pv, Shared& S) {
  const double thr = __dsub_rn(1.0, (double)p);
  double sum = 0.0;
  for (int base = 0; base < n; base += NT) {
    const int e = base + threadIdx.x;
    if (e < n) pv[threadIdx.x] = prob(srow[ckey_idx(K[e])], m);
    csync();
    if (threadIdx.x == 0) {
      const int lim = min(NT, n - base);
      for (int j = 0; j < lim; ++j) sum = __dadd_rn(sum, pv[j]);
    }
    csync();
  }
  if (threadIdx.x == 0) { S.dsum = sum; S.jstar = n; }
  csync();
  sum = S.dsum;
  double cum = 0.0;
  for (int base = 0; base < n; base += NT) {
    const int e = base + threadIdx.x;
    if (e < n) pv[threadIdx.x] = __ddiv_rn(prob(srow[ckey_idx(K[e])], m), sum);
    csync();
    if (threadIdx.x == 0) {
      const int lim = min(NT, n - base);
      for (int j = 0; j < lim; ++j) {
        cum = __dadd_rn(cum, pv[j]);
        if (!(cum <= thr)) { S.jstar = base + j; break; }
      }
    }
    csync();
    if (S.jstar < n) break;
  }
  const int js = S.jstar;
  csync();
  return js;
}

// Exact reference top-p sums over the list when pv[0..n) already holds the
// probabilities in ascending order (n <= LIST_CAP). Returns the crossing.
__device__ int topp_exact_pv(int n, float p, double* pv, Shared& S) {
  const double thr = __dsub_rn(1.0, (double)p);
  if (threadIdx.x == 0) {
    double sum = 0.0;
    for (int e = 0; e < n; ++e) sum = __dadd_rn(sum, pv[e]);
    S.dsum = sum;
  }
  csync();
  const double sum = S.dsum;
  for (int e = threadIdx.x; e < n; e += NT) pv[e] = __ddiv_rn(pv[e], sum);
  csync();
  if (threadIdx.x == 0) {
    double cum = 0.0;
    int js = n;
    for (int e = 0; e < n; ++e) {
      cum = __dadd_rn(cum, pv[e]);
      if (!(cum <= thr)) { js = e; break; }
    }
    S.jstar = js;
  }
  csync();
  const int js = S.jstar;
  csync();
  return js;
}

// Top-p over the survivor list K[0..n) (sorted ascending). Returns K*.
__device__ unsigned long long topp_list(const Args& a, const float* srow, const unsigned long long* K, int n,
                                        float m, const c4s_row_params& P, double* pv, Shared& S) {
  if (n <= 0) return 0ull;
  const double thr = __dsub_rn(1.0, (double)P.top_p);
  for (int e = threadIdx.x; e < n; e += NT) pv[e] = prob(srow[ckey_idx(K[e])], m);
  csync();
  bool exact = (n <= SEQ_MAX) || (a.debug & C4S_DEBUG_FORCE_EXACT);
  int jstar = n;
  if (!exact) {
    // Fixed-point prefix sums: thread t owns entries [t*E, t*E+E).
    const int E = (n + NT - 1) / NT;
    const int lo = min(n, threadIdx.x * E), hi = min(n, lo + E);
    unsigned long long loc = 0;
    for (int e = lo; e < hi; ++e) loc += qfix(pv[e], a.qscale);
    unsigned long long SQ;
    const unsigned long long base = block_exscan_u64(loc, S.red64, &SQ);
    const double SQd = (double)SQ, Tq = __dmul_rn(thr, SQd), bq = band_q(n, SQd);
    if (threadIdx.x == 0) { S.jstar = n; S.u64a = SQ; S.u64b = 0; }
    csync();
    unsigned long long run = base;
    for (int e = lo; e < hi; ++e) {
      const unsigned long long q = qfix(pv[e], a.qscale);
      if ((double)(run + q) > Tq) {
        atomicMin(&S.jstar, e);
        break;
      }
      run += q;
    }
    csync();
    jstar = S.jstar;
    if (jstar < n && lo <= jstar && jstar < hi) {
      unsigned long long r = base;
      for (int e = lo; e < jstar; ++e) r += qfix(pv[e], a.qscale);
      S.u64a = r;
      S.u64b = r + qfix(pv[jstar], a.qscale);
    }
    csync();
    const bool ok = SQ > 0 && (double)S.u64a <= Tq - bq && (jstar == n || (double)S.u64b > Tq + bq);
    csync();
    if (!ok) {
      exact = true;
      if (threadIdx.x == 0) atomicAdd(&a.counters[C4S_CNT_TOPP_EXACT_FALLBACK], 1ull);
    }
  }
  if (exact) jstar = topp_exact_pv(n, P.top_p, pv, S);
  const unsigned long long Kp = (jstar < n) ? K[jstar] : KEY_MAX;
  const int mk = P.min_tokens_to_keep;
  const unsigned long long Kkeep = (mk <= 0) ? KEY_MAX : (mk <= n ? K[n - mk] : 0ull);
  return Kp < Kkeep ? Kp : Kkeep;
}

// Exact top-p over all survivors via a bitonic sort of the row's keys in the
// CTA's global scratch slab (rare fallback for large candidate sets).
__device__ unsigned long long topp_global(const Args& a, const float* srow, float m, float thresh,
                                          const c4s_row_params& P, double* pv, Shared& S) {
  const int V = a.V;
  unsigned long long* G = a.scratch + (size_t)blockIdx.x * (size_t)a.scratch_stride;
  const int P2 = next_pow2(V);
  int cl = 0;
  for (int i = threadIdx.x; i < P2; i += NT) {
    unsigned long long k = KEY_MAX;
    if (i < V) {
      const float y = srow[i];
      if (y > -INFINITY && y >= thresh) { k = ckey(y, i); ++cl; }
    }
    G[i] = k;
  }
  const int n = block_reduce(cl, SumI(), S.redi);
  bitonic_sort_u64(G, P2);
  if (n == 0) return 0ull;
  const int jstar = topp_exact_seq(srow, G, n, m, P.top_p, pv, S);
  const unsigned long long Kp = (jstar < n) ? G[jstar] : KEY_MAX;
  const int mk = P.min_tokens_to_keep;
  const unsigned long long Kkeep = (mk <= 0) ? KEY_MAX : (mk <= n ? G[n - mk] : 0ull);
  csync();
  return Kp < Kkeep ? Kp : Kkeep;
}

// Top-p over many survivors: probability mass per distance-from-max bin,
// then the crossing bin's elements sorted in shared memory.
__device__ unsigned long long topp_binned(const Args& a, const float* srow, float m, float thresh,
                                          const c4s_row_params& P, unsigned* cnt, unsigned long long* mass,
                                          unsigned long long* lkey, double* pv, Shared& S) {
  const int V = a.V;
  const double thr = __dsub_rn(1.0, (double)P.top_p);
  if ((a.debug & C4S_DEBUG_FORCE_EXACT) || P.min_tokens_to_keep > 1 || !(m < INFINITY))
    return topp_global(a, srow, m, thresh, P, pv, S);
  for (int j = threadIdx.x; j < NBIN; j += NT) { cnt[j] = 0; mass[j] = 0; }
  csync();
  unsigned long long kmax = 0;
  for (int i = threadIdx.x; i < V; i += NT) {
    const float y = srow[i];
    if (y > -INFINITY && y >= thresh) {
      const int b = vbin(m, y);
      atomicAdd(&mass[b], qfix(prob(y, m), a.qscale));
      atomicAdd(&cnt[b], 1u);
      const unsigned long long k = ckey(y, i);
      kmax = k > kmax ? k : kmax;
    }
  }
  kmax = block_reduce(kmax, MaxU64(), S.red64);  // syncs: bins are complete
  static_assert(NT == NBIN, "one bin per thread");
  const unsigned long long sq = block_reduce(mass[threadIdx.x], SumU64(), S.red64);
  const int ns = block_reduce((int)cnt[threadIdx.x], SumI(), S.redi);
  if (ns == 0) return 0ull;
  const unsigned long long Kkeep = (P.min_tokens_to_keep <= 0) ? KEY_MAX : kmax;
  const double SQd = (double)sq, Tq = __dmul_rn(thr, SQd), bq = band_q(ns, SQd);
  if (thr < 0.0) return 0ull;                 // p > 1: cum > 1-p everywhere, nothing removed
  if (thr == 0.0) {
    // p == 1: cum stays exactly 0 only across zero probabilities, so exactly
    // the survivors whose exp() underflows to 0 are removed.
    unsigned long long kmin = KEY_MAX;
    for (int i = threadIdx.x; i < V; i += NT) {
      const float y = srow[i];
      if (y > -INFINITY && y >= thresh && prob(y, m) > 0.0) {
        const unsigned long long k = ckey(y, i);
        kmin = k < kmin ? k : kmin;
      }
    }
    kmin = block_reduce(kmin, [](unsigned long long x, unsigned long long y) { return x < y ? x : y; }, S.red64);
    return kmin < Kkeep ? kmin : Kkeep;
  }
  if (Tq >= SQd - a.qscale) {
    // The crossing, if any, is at the largest element (probability 1 = qscale
    // units), which min_tokens_to_keep >= 1 keeps: everything else is removed
    // once the mass below it is certainly <= 1-p.
    if (P.min_tokens_to_keep >= 1 && SQd - a.qscale <= Tq - bq) return Kkeep;
    if (P.min_tokens_to_keep <= 0 && SQd <= Tq - bq) return Kkeep;
    if (Tq >= SQd) {
      if (threadIdx.x == 0) atomicAdd(&a.counters[C4S_CNT_TOPP_EXACT_FALLBACK], 1ull);
      return topp_global(a, srow, m, thresh, P, pv, S);
    }
  }
  const unsigned long long target = (unsigned long long)floor(Tq);
  // ascending value order = descending bin index
  if (threadIdx.x < 32)
    warp_find_bin<unsigned long long>([&](int j) { return mass[255 - j]; }, target, true, &S.c, &S.mbefore);
  csync();
  const int c = 255 - S.c;  // S.c < NBIN because target < sq
  const unsigned long long before = S.mbefore;
  const int nc = (int)cnt[c];
  csync();
  if (nc > LIST_CAP) {
    if (threadIdx.x == 0) atomicAdd(&a.counters[C4S_CNT_TOPP_EXACT_FALLBACK], 1ull);
    return topp_global(a, srow, m, thresh, P, pv, S);
  }
  const int n = gather_sort(srow, V, lkey, S,
                            [&](float y, int) { return y > -INFINITY && y >= thresh && vbin(m, y) == c; }, false);
  // prefix over the sorted bin (thread t owns entries [t*E, t*E+E))
  const int E = (n + NT - 1) / NT;
  const int lo = threadIdx.x * E, hi = min(n, lo + E);
  unsigned long long loc = 0;
  for (int e = lo; e < hi; ++e) loc += qfix(prob(srow[ckey_idx(lkey[e])], m), a.qscale);
  unsigned long long tot;
  const unsigned long long pbase = before + block_exscan_u64(loc, S.red64, &tot);
  if (threadIdx.x == 0) { S.jstar = n; S.u64a = before; S.u64b = 0; }
  csync();
  unsigned long long run = pbase;
  for (int e = lo; e < hi; ++e) {
    const unsigned long long q = qfix(prob(srow[ckey_idx(lkey[e])], m), a.qscale);
    if ((double)(run + q) > Tq) { atomicMin(&S.jstar, e); break; }
    run += q;
  }
  csync();
  const int jstar = S.jstar;
  if (jstar < n && lo <= jstar && jstar < hi) {
    unsigned long long r = pbase;
    for (int e = lo; e < jstar; ++e) r += qfix(prob(srow[ckey_idx(lkey[e])], m), a.qscale);
    S.u64a = r;
    S.u64b = r + qfix(prob(srow[ckey_idx(lkey[jstar])], m), a.qscale);
  }
  csync();
  const bool ok = jstar < n && (double)S.u64a <= Tq - bq && (double)S.u64b > Tq + bq;
  const unsigned long long Kp = jstar < n ? lkey[jstar] : KEY_MAX;
  csync();
  if (!ok) {
    if (threadIdx.x == 0) atomicAdd(&a.counters[C4S_CNT_TOPP_EXACT_FALLBACK], 1ull);
    return topp_global(a, srow, m, thresh, P, pv, S);
  }
  return Kp < Kkeep ? Kp : Kkeep;
}

// Exact reference draw over the index-sorted survivor list I[0..n)
// (text2semantic.cpp:150-165), by one thread.
__device__ int draw_exact_list(const float* srow, const unsigned long long* I, int n, float md, double u,
                               int V, const double* pv, Shared& S) {
  if (threadIdx.x == 0) {
    double sum = 0.0;
    for (int e = 0; e < n; ++e) sum = __dadd_rn(sum, pv[e]);
    const double r = __dmul_rn(u, sum);
    int tok = V - 1;
    if (r == 0.0) {
      tok = 0;
    } else {
      double acc = 0.0;
      for (int e = 0; e < n; ++e) {
        acc = __dadd_rn(acc, pv[e]);
        if (r <= acc) { tok = (int)I[e]; break; }
      }
    }
    S.tok = tok;
  }
  csync();
  const int t = S.tok;
  csync();
  return t;
}

// Exact reference draw by chunked sequential sums over the whole row.
template <typename Pred>
__device__ int draw_exact_row(const float* srow, int V, float md, double u, double* pv, Shared& S, Pred D) {
  double sum = 0.0;
  for (int base = 0; base < V; base += NT) {
    const int i = base + threadIdx.x;
    double p = 0.0;
    if (i < V) { const float y = srow[i]; if (D(y, i)) p = prob(y, md); }
    pv[threadIdx.x] = p;
    csync();
    if (threadIdx.x == 0) {
      const int lim = min(NT, V - base);
      for (int j = 0; j < lim; ++j) if (pv[j] != 0.0) sum = __dadd_rn(sum, pv[j]);
    }
    csync();
  }
  if (threadIdx.x == 0) { S.dsum = __dmul_rn(u, sum); S.tok = (S.dsum == 0.0) ? 0 : -1; }
  csync();
  const double r = S.dsum;
  double acc = 0.0;
  for (int base = 0; base < V && S.tok < 0; base += NT) {
    const int i = base + threadIdx.x;
    double p = 0.0;
    if (i < V) { const float y = srow[i]; if (D(y, i)) p = prob(y, md); }
    pv[threadIdx.x] = p;
    csync();
    if (threadIdx.x == 0) {
      const int lim = min(NT, V - base);
      for (int j = 0; j < lim; ++j) {
        if (pv[j] == 0.0) continue;
        acc = __dadd_rn(acc, pv[j]);
        if (r <= acc) { S.tok = base + j; break; }
      }
    }
    csync();
  }
  if (threadIdx.x == 0 && S.tok < 0) S.tok = V - 1;
  csync();
  const int t = S.tok;
  csync();
  return t;
}

// Draw over the index-sorted survivor list I[0..n); pv gets the probabilities.
__device__ int draw_list(const Args& a, const float* srow, const unsigned long long* I, int n, float md,
                         double u, double* pv, Shared& S) {
  for (int e = threadIdx.x; e < n; e += NT) pv[e] = prob(srow[(int)I[e]], md);
  csync();
  if (n <= SEQ_MAX || (a.debug & C4S_DEBUG_FORCE_EXACT) || n == 0)
    return n == 0 ? 0 : draw_exact_list(srow, I, n, md, u, a.V, pv, S);
  const int E = (n + NT - 1) / NT;
  const int lo = threadIdx.x * E, hi = min(n, lo + E);
  unsigned long long loc = 0;
  for (int e = lo; e < hi; ++e) loc += qfix(pv[e], a.qscale);
  unsigned long long SQ;
  const unsigned long long base = block_exscan_u64(loc, S.red64, &SQ);
  const double SQd = (double)SQ, rq = __dmul_rn(u, SQd), bq = band_q(n, SQd);
  if (threadIdx.x == 0) { S.jstar = n; S.u64a = 0; S.u64b = 0; }
  csync();
  unsigned long long run = base;
  for (int e = lo; e < hi; ++e) {
    const unsigned long long q = qfix(pv[e], a.qscale);
    if ((double)(run + q) >= rq) {
      atomicMin(&S.jstar, e);
      break;
    }
    run += q;
  }
  csync();
  const int js = S.jstar;
  if (js < n && lo <= js && js < hi) {
    unsigned long long r = base;
    for (int e = lo; e < js; ++e) r += qfix(pv[e], a.qscale);
    S.u64a = r;
    S.u64b = r + qfix(pv[js], a.qscale);
  }
  csync();
  const bool ok = SQ > 0 && js < n && (double)S.u64a < rq - bq && (double)S.u64b > rq + bq;
  csync();
  if (ok) return (int)I[js];
  if (threadIdx.x == 0) atomicAdd(&a.counters[C4S_CNT_DRAW_EXACT_FALLBACK], 1ull);
  return draw_exact_list(srow, I, n, md, u, a.V, pv, S);
}

// Draw over more survivors than the list holds: fixed-point prefix over the
// row with each thread owning a contiguous index range (odd stride: no bank
// conflicts), exact chunked fallback.
template <typename Pred>
__device__ int draw_rowpass(const Args& a, const float* srow, float md, double u, double* pv, Shared& S,
                            Pred D) {
  const int V = a.V;
  if (a.debug & C4S_DEBUG_FORCE_EXACT) return draw_exact_row(srow, V, md, u, pv, S, D);
  int C = (V + NT - 1) / NT;
  if (!(C & 1)) ++C;
  const int lo = min(V, threadIdx.x * C), hi = min(V, lo + C);
  unsigned long long loc = 0;
  int nl = 0;
  for (int i = lo; i < hi; ++i) {
    const float y = srow[i];
    if (D(y, i)) { loc += qfix(prob(y, md), a.qscale); ++nl; }
  }
  unsigned long long SQ;
  const unsigned long long base = block_exscan_u64(loc, S.red64, &SQ);
  const int n = block_reduce(nl, SumI(), S.redi);
  const double SQd = (double)SQ, rq = __dmul_rn(u, SQd), bq = band_q(n, SQd);
  if (threadIdx.x == 0) { S.tok = -1; S.u64a = 0; S.u64b = 0; }
  csync();
  if (SQ > 0 && (double)base < rq && (double)(base + loc) >= rq) {
    unsigned long long run = base;
    for (int i = lo; i < hi; ++i) {
      const float y = srow[i];
      if (!D(y, i)) continue;
      const unsigned long long q = qfix(prob(y, md), a.qscale);
      if ((double)(run + q) >= rq) { S.tok = i; S.u64a = run; S.u64b = run + q; break; }
      run += q;
    }
  }
  csync();
  const int tok = S.tok;
  const bool ok = tok >= 0 && (double)S.u64a < rq - bq && (double)S.u64b > rq + bq;
  csync();
  if (ok) return tok;
  if (threadIdx.x == 0) atomicAdd(&a.counters[C4S_CNT_DRAW_EXACT_FALLBACK], 1ull);
  return draw_exact_row(srow, V, md, u, pv, S, D);
}

// ---------------------------------------------------------------------------
// Row staging shared by both kernels.
// ---------------------------------------------------------------------------
struct Stage {
  int shift;  // smem offset of element 0 inside the row buffer (0..3)
  int body;   // elements moved by the bulk copy (0: nothing in flight)
};

// Issue the staging of one row: the 16-byte-aligned body with one bulk-async
// copy completing on `bar`, the unaligned head and tail (<= 3 elements each)
// with plain loads. Thread 0 issues the copy; every thread must call.
__device__ __forceinline__ Stage stage_issue(const float* g, int V, float* rowbuf, unsigned long long* bar) {
  const unsigned long long ga = (unsigned long long)g;
  int head = (int)(((16u - (unsigned)(ga & 15ull)) & 15u) >> 2);
  if (head > V) head = V;
  const int body = ((V - head) >> 2) << 2;
  const int shift = (4 - head) & 3;
  float* srow = rowbuf + shift;
  if (threadIdx.x == 0 && body > 0) {
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(bar, (unsigned)body * 4u);
    bulk_g2s(srow + head, g + head, (unsigned)body * 4u, bar);
  }
  for (int i = threadIdx.x; i < head; i += NT) srow[i] = g[i];
  for (int i = head + body + threadIdx.x; i < V; i += NT) srow[i] = g[i];
  return Stage{shift, body};
}

// Bounded wait for a staged row (thread 0 polls, then a CTA barrier).
// Returns false on every thread if the wait gave up.
__device__ __forceinline__ bool stage_wait(const Args& a, const Stage& st, unsigned long long* bar,
                                           unsigned& phase, Shared& S) {
  if (threadIdx.x == 0) {
    bool ok = true;
    if (st.body > 0) ok = mbar_wait_bounded(bar, phase);
    S.abort_row = ok ? 0 : 1;
    if (!ok) atomicOr(a.errflags, C4S_DEVERR_TIMEOUT);
  }
  if (st.body > 0) phase ^= 1u;
  csync();
  return S.abort_row == 0;
}

// Validated history window [h0, h1) of a row (empty if the penalty is off).
__device__ __forceinline__ void hist_window(const Args& a, int row, bool do_pen, long long& h0, long long& h1) {
  h0 = h1 = 0;
  if (!do_pen) return;
  h0 = a.hist_off[row];
  h1 = a.hist_len ? h0 + a.hist_len[row] : a.hist_off[row + 1];
  if (h0 < 0 || h1 < h0 || h1 > a.hist_total) {
    if (threadIdx.x == 0) atomicOr(a.errflags, C4S_DEVERR_HIST_RANGE);
    h0 = h1 = 0;
  }
}

// First 8*NT history ids of a row into registers (-1 = none).
__device__ __forceinline__ void hist_prefetch(const Args& a, long long h0, long long h1, int (&hid)[8]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const long long j = h0 + threadIdx.x + (long long)q * NT;
    hid[q] = (j < h1) ? a.hist[j] : -1;
  }
}

// Repetition penalty (sampling.cpp:19-28): each distinct in-range id once,
// de-duplicated by a zeroed shared bitmap. Ends with a CTA barrier.
__device__ __forceinline__ void penalty_apply(const Args& a, float* srow, int V, unsigned* bitmap, float pen,
                                              const int (&hid)[8], long long h0, long long h1) {
  const float rpen = __frcp_rn(pen);
  auto apply = [&](int t) {
    if ((unsigned)t < (unsigned)V) {
      const unsigned bit = 1u << (t & 31);
      const unsigned old = atomicOr(&bitmap[t >> 5], bit);
      if (!(old & bit)) {
        const float s = srow[t];
        srow[t] = (s < 0.0f) ? __fmul_rn(s, pen) : div_rn(s, pen, rpen);
      }
    }
  };
#pragma unroll
  for (int q = 0; q < 8; ++q) apply(hid[q]);
  for (long long j = h0 + threadIdx.x + 8LL * NT; j < h1; j += NT) apply(a.hist[j]);
  csync();
}

// ---------------------------------------------------------------------------
// General (exact) processing of one staged, penalised row: greedy argmax, or
// temperature, top-k, top-p, draw; then the id and, on request, the
// processed logits. Handles every vocabulary size up to MAX_VOCAB and every
// input the reference defines.
// ---------------------------------------------------------------------------
__device__ __noinline__ void finish_general(const Args& a, int row, const c4s_row_params& P, int st, float* srow,
                               unsigned* cnt, unsigned long long* mass, unsigned long long* lkey, double* pv,
                               Shared& S) {
  const int V = a.V;
  const int tid = threadIdx.x;
  const bool sample = a.mode == MODE_SAMPLE;
  // ---- 3a. greedy / argmax ----------------------------------------------------
  if (a.mode == MODE_ARGMAX || (sample && P.greedy)) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = tid; i < V; i += NT) {
      const float v = srow[i];
      if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(FULL, bv, o);
      const int oi = __shfl_xor_sync(FULL, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if ((tid & 31) == 0) { S.redf[tid >> 5] = bv; S.redi[tid >> 5] = bi; }
    csync();
    if (tid == 0) {
      float b = S.redf[0];
      int ix = S.redi[0];
      for (int w = 1; w < NWARP; ++w)
        if (S.redf[w] > b || (S.redf[w] == b && S.redi[w] < ix)) { b = S.redf[w]; ix = S.redi[w]; }
      a.out_ids[row] = ix;
    }
    if (sample && a.out_logits) {
      float* o = a.out_logits + (long long)row * a.out_ld;
      for (int i = tid; i < V; i += NT) o[i] = srow[i];
    }
    csync();
    return;
  }

  // ---- 3b. temperature + row max -----------------------------------------------
  const float T = P.temperature;
  const bool do_t = (st & C4S_STAGE_TEMPERATURE) && !(T == 1.0f || T <= 0.0f);
  float lmax = -INFINITY;
  for (int i = tid; i < V; i += NT) {
    float y = srow[i];
    if (do_t) { y = __fdiv_rn(y, T); srow[i] = y; }
    lmax = fmaxf(lmax, y);
  }
  const float m = block_reduce(lmax, MaxF(), S.redf);

  // ---- 3c. top-k threshold ------------------------------------------------------
  const bool do_k = (st & C4S_STAGE_TOP_K) && P.top_k > 0 && P.top_k < V;
  const bool do_p = (st & C4S_STAGE_TOP_P) != 0;
  float thresh = -INFINITY;
  int n_list = -1, lbase = 0;
  if (do_k) {
    bool done = false;
    if (!(a.debug & C4S_DEBUG_FORCE_EXACT) && m > -INFINITY && m < INFINITY) {
      for (int j = tid; j < NBIN; j += NT) cnt[j] = 0;
      csync();
      for (int i = tid; i < V; i += NT) {
        const int b = vbin(m, srow[i]);
        if (b < NBIN - 1) atomicAdd(&cnt[b], 1u);
      }
      csync();
      if (tid < 32)
        warp_find_bin<unsigned>([&](int j) { return cnt[j]; }, (unsigned)P.top_k, false, &S.c, &S.cbefore);
      csync();
      const int c = S.c;
      const int nle = (c < NBIN - 1) ? (int)(S.cbefore + cnt[c]) : LIST_CAP + 1;
      csync();
      if (nle <= LIST_CAP) {
        const int n = gather_sort(srow, V, lkey, S, [&](float y, int) { return vbin(m, y) <= c; }, false);
        thresh = fkey_inv((unsigned)(lkey[n - P.top_k] >> 32));
        const unsigned tk = fkey(thresh);
        int below = 0;
        for (int e = tid; e < n; e += NT) below += ((unsigned)(lkey[e] >> 32) < tk) ? 1 : 0;
        below = block_reduce(below, SumI(), S.redi);
        lbase = below;
        n_list = n - below;
        done = true;
      }
    }
    if (!done) {
      thresh = radix_kth_largest(srow, V, P.top_k, cnt, S);
      if (tid == 0) atomicAdd(&a.counters[C4S_CNT_TOPK_RADIX], 1ull);
    }
  }
  const float thr_k = thresh;
  auto surv = [thr_k](float y) { return y > -INFINITY && y >= thr_k; };

  // ---- 3d. top-p ----------------------------------------------------------------
  unsigned long long kstar = 0ull;
  if (do_p) {
    if (n_list < 0 && !(a.debug & C4S_DEBUG_FORCE_BINS)) {
      int cl = 0;
      for (int i = tid; i < V; i += NT) cl += surv(srow[i]) ? 1 : 0;
      const int ns = block_reduce(cl, SumI(), S.redi);
      if (ns <= LIST_CAP) {
        n_list = gather_sort(srow, V, lkey, S, [&](float y, int) { return surv(y); }, false);
        lbase = 0;
      }
    }
    if (n_list >= 0 && !(a.debug & C4S_DEBUG_FORCE_BINS)) {
      kstar = topp_list(a, srow, lkey + lbase, n_list, m, P, pv, S);
    } else {
      if (tid == 0) atomicAdd(&a.counters[C4S_CNT_TOPP_BINNED], 1ull);
      kstar = topp_binned(a, srow, m, thresh, P, cnt, mass, lkey, pv, S);
    }
  }
  const unsigned long long ks = kstar;
  auto keep = [thr_k, ks](float y, int i) { return y > -INFINITY && y >= thr_k && ckey(y, i) >= ks; };

  // ---- 3e. draw ------------------------------------------------------------------
  if (sample) {
    const float md = fmaxf(-1e30f, m);
    if (tid == 0) {
      unsigned long long x = a.rng[row];
      x ^= x << 13; x ^= x >> 7; x ^= x << 17;
      a.rng[row] = x;
      S.u64c = x >> 11;
    }
    csync();
    const unsigned long long u53 = S.u64c;
    const double u = (double)u53 * 1.1102230246251565e-16;  // (x>>11) / 2^53, exact
    int tok;
    if (u53 == 0ull) {
      tok = 0;
    } else if (n_list >= 0 && !(a.debug & C4S_DEBUG_FORCE_BINS)) {
      // survivors after top-p are the list suffix with key >= K*
      const unsigned long long* K = lkey + lbase;
      int cb = 0;
      for (int e = tid; e < n_list; e += NT) cb += (K[e] < ks) ? 1 : 0;
      const int jf = block_reduce(cb, SumI(), S.redi);
      const int nk = n_list - jf;
      unsigned long long tmp[LIST_CAP / NT];
#pragma unroll
      for (int q = 0; q < LIST_CAP / NT; ++q) {
        const int e = tid + q * NT;
        tmp[q] = (e < nk) ? (unsigned long long)ckey_idx(K[jf + e]) : KEY_MAX;
      }
      csync();
      const int np = next_pow2(max(nk, 1));
#pragma unroll
      for (int q = 0; q < LIST_CAP / NT; ++q) {
        const int e = tid + q * NT;
        if (e < np) lkey[e] = tmp[q];
      }
      csync();
      bitonic_sort_u64(lkey, np);
      tok = draw_list(a, srow, lkey, nk, md, u, pv, S);
    } else {
      int cl = 0;
      for (int i = tid; i < V; i += NT) cl += keep(srow[i], i) ? 1 : 0;
      const int nk = block_reduce(cl, SumI(), S.redi);
      if (nk <= LIST_CAP && !(a.debug & C4S_DEBUG_FORCE_BINS)) {
        const int n = gather_sort(srow, V, lkey, S, keep, true);
        tok = draw_list(a, srow, lkey, n, md, u, pv, S);
      } else {
        if (tid == 0) atomicAdd(&a.counters[C4S_CNT_DRAW_ROWPASS], 1ull);
        tok = draw_rowpass(a, srow, md, u, pv, S, keep);
      }
    }
    if (tid == 0) a.out_ids[row] = tok;
  }

  // ---- 4. processed logits ---------------------------------------------------------
  float* out = nullptr;
  if (a.mode == MODE_PROCESS) out = a.inout + (long long)row * a.ld;
  else if (sample && a.out_logits) out = a.out_logits + (long long)row * a.out_ld;
  if (out) {
    for (int i = tid; i < V; i += NT) {
      const float y = srow[i];
      const bool masked = (y < thr_k) || (y > -INFINITY && ckey(y, i) < ks);
      out[i] = masked ? -INFINITY : y;
    }
  }
}

// One row through the general path from global memory: stage, penalty,
// finish_general. Returns false if the staging wait gave up.
__device__ __noinline__ bool general_row(const Args& a, int row, float* rowbuf, unsigned* bitmap, unsigned* cnt,
                            unsigned long long* mass, unsigned long long* lkey, double* pv, Shared& S,
                            unsigned& phase) {
  const int V = a.V;
  const c4s_row_params P = a.params[(long long)row * a.params_stride];
  const int st = a.mode == MODE_SAMPLE
                     ? (C4S_STAGE_PENALTY | C4S_STAGE_TEMPERATURE | C4S_STAGE_TOP_K | C4S_STAGE_TOP_P)
                     : (a.mode == MODE_PROCESS ? a.stages : 0);
  const float* g = (a.mode == MODE_PROCESS ? a.inout : a.logits) + (long long)row * a.ld;
  const Stage sg = stage_issue(g, V, rowbuf, &S.bar);
  const bool pen = (st & C4S_STAGE_PENALTY) && a.hist_off && P.repetition_penalty != 1.0f;
  long long h0, h1;
  hist_window(a, row, pen, h0, h1);
  int hid[8];
  hist_prefetch(a, h0, h1, hid);
  if (pen)
    for (int w = threadIdx.x; w < (V + 31) / 32; w += NT) bitmap[w] = 0u;
  if (!stage_wait(a, sg, &S.bar, phase, S)) return false;
  float* srow = rowbuf + sg.shift;
  if (pen) penalty_apply(a, srow, V, bitmap, P.repetition_penalty, hid, h0, h1);
  finish_general(a, row, P, st, srow, cnt, mass, lkey, pv, S);
  csync();
  return true;
}

}  // namespace c4s
