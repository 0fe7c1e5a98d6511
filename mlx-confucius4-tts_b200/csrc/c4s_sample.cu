// c4s_sample.cu -- sm_100a kernels and C ABI of the T2S sampling stage.
//
// One persistent CTA processes one logits row at a time (rows r = blockIdx.x,
// blockIdx.x + gridDim.x, ...). Per row:
//   1. stage the row into shared memory: the 16-byte-aligned body with one
//      bulk-async copy (TMA engine, mbarrier completion), the <= 3-element
//      unaligned head and tail with plain loads; history ids are fetched into
//      registers while the copy is in flight;
//   2. repetition penalty: scatter over the history, de-duplicated with a
//      shared-memory bitmap (sampling.cpp:19-28 of the reference);
//   3. greedy rows: block argmax (sampling.cpp:73-76);
//      sample rows: temperature + row max in one pass (sampling.cpp:14-17),
//      top-k threshold by a 256-bin distance-from-max histogram, a gather of
//      the few candidate bins and a shared-memory sort (exact order statistic,
//      sampling.cpp:30-40), top-p and the draw (sampling.cpp:42-71,
//      text2semantic.cpp:150-165) as described below;
//   4. write the id (and, on request, the processed logits).
//
// Exactness of top-p and the draw. The reference sums exp() in double, in a
// fixed order (ascending value for top-p, index order for the draw). With at
// most SEQ_MAX survivors one thread repeats that sequential sum exactly. With
// more survivors, the CTA computes the same prefix sums in 64-bit fixed point
// (order independent), locates the crossing element, and accepts it only if
// the crossing is farther from the threshold than a proven bound on the
// difference between the fixed-point estimate and the reference's rounded
// sequential sum. Otherwise (probability ~1e-7 per row) it falls back to the
// exact sequential sum: over the sorted candidate list in shared memory, or,
// for very large candidate sets, after a bitonic sort of the row's keys in
// a per-CTA global scratch slab.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/c4s_sampling.h"
#include "c4s_device.cuh"

namespace c4s {

enum { MODE_SAMPLE = 0, MODE_PROCESS = 1, MODE_ARGMAX = 2 };

struct Args {
  const float* logits;          // MODE_SAMPLE / MODE_ARGMAX input
  float* inout;                 // MODE_PROCESS rows (in place)
  int B, V;
  long long ld;
  const int* hist;
  const long long* hist_off;
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
  unsigned long long u64a, u64b, u64c;
  double dsum;
  int c, slot, jstar, tok, abort_row;
  unsigned cbefore;
  unsigned long long mbefore;
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

__device__ __forceinline__ double prob(float y, float m) {
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
    __syncthreads();
    for (int i = threadIdx.x; i < V; i += NT) {
      const unsigned u = fkey(srow[i]);
      if ((u & pmask) == prefix) atomicAdd(&cnt[(u >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x < 32)
      warp_find_bin<unsigned>([&](int j) { return cnt[255 - j]; }, kk, false, &S.c, &S.cbefore);
    __syncthreads();
    const unsigned d = 255u - (unsigned)S.c;
    kk -= S.cbefore;
    prefix |= d << shift;
    pmask |= 0xffu << shift;
    __syncthreads();
  }
  return fkey_inv(prefix);
}

// Gather keys ckey(y,i) of all elements with pred(y, i) into lkey[0..n), pad to
// a power of two and sort ascending. Returns n (caller guarantees n <= LIST_CAP).
template <typename Pred>
__device__ int gather_sort(const float* srow, int V, unsigned long long* lkey, Shared& S, Pred pred,
                           bool index_keys) {
  if (threadIdx.x == 0) S.slot = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < V; i += NT) {
    const float y = srow[i];
    if (pred(y, i)) {
      const int s = atomicAdd(&S.slot, 1);
      if (s < LIST_CAP) lkey[s] = index_keys ? (unsigned long long)i : ckey(y, i);
    }
  }
  __syncthreads();
  const int n = min(S.slot, LIST_CAP);
  const int np = next_pow2(max(n, 1));
  for (int p = n + threadIdx.x; p < np; p += NT) lkey[p] = KEY_MAX;
  __syncthreads();
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
    __syncthreads();
    if (threadIdx.x == 0) {
      const int lim = min(NT, n - base);
      for (int j = 0; j < lim; ++j) sum = __dadd_rn(sum, pv[j]);
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) { S.dsum = sum; S.jstar = n; }
  __syncthreads();
  sum = S.dsum;
  double cum = 0.0;
  for (int base = 0; base < n; base += NT) {
    const int e = base + threadIdx.x;
    if (e < n) pv[threadIdx.x] = __ddiv_rn(prob(srow[ckey_idx(K[e])], m), sum);
    __syncthreads();
    if (threadIdx.x == 0) {
      const int lim = min(NT, n - base);
      for (int j = 0; j < lim; ++j) {
        cum = __dadd_rn(cum, pv[j]);
        if (!(cum <= thr)) { S.jstar = base + j; break; }
      }
    }
    __syncthreads();
    if (S.jstar < n) break;
  }
  const int js = S.jstar;
  __syncthreads();
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
  __syncthreads();
  const double sum = S.dsum;
  for (int e = threadIdx.x; e < n; e += NT) pv[e] = __ddiv_rn(pv[e], sum);
  __syncthreads();
  if (threadIdx.x == 0) {
    double cum = 0.0;
    int js = n;
    for (int e = 0; e < n; ++e) {
      cum = __dadd_rn(cum, pv[e]);
      if (!(cum <= thr)) { js = e; break; }
    }
    S.jstar = js;
  }
  __syncthreads();
  const int js = S.jstar;
  __syncthreads();
  return js;
}

// Top-p over the survivor list K[0..n) (sorted ascending). Returns K*.
__device__ unsigned long long topp_list(const Args& a, const float* srow, const unsigned long long* K, int n,
                                        float m, const c4s_row_params& P, double* pv, Shared& S) {
  if (n <= 0) return 0ull;
  const double thr = __dsub_rn(1.0, (double)P.top_p);
  for (int e = threadIdx.x; e < n; e += NT) pv[e] = prob(srow[ckey_idx(K[e])], m);
  __syncthreads();
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
    __syncthreads();
    unsigned long long run = base;
    for (int e = lo; e < hi; ++e) {
      const unsigned long long q = qfix(pv[e], a.qscale);
      if ((double)(run + q) > Tq) {
        atomicMin(&S.jstar, e);
        break;
      }
      run += q;
    }
    __syncthreads();
    jstar = S.jstar;
    if (jstar < n && lo <= jstar && jstar < hi) {
      unsigned long long r = base;
      for (int e = lo; e < jstar; ++e) r += qfix(pv[e], a.qscale);
      S.u64a = r;
      S.u64b = r + qfix(pv[jstar], a.qscale);
    }
    __syncthreads();
    const bool ok = SQ > 0 && (double)S.u64a <= Tq - bq && (jstar == n || (double)S.u64b > Tq + bq);
    __syncthreads();
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
  __syncthreads();
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
  __syncthreads();
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
  __syncthreads();
  const int c = 255 - S.c;  // S.c < NBIN because target < sq
  const unsigned long long before = S.mbefore;
  const int nc = (int)cnt[c];
  __syncthreads();
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
  __syncthreads();
  unsigned long long run = pbase;
  for (int e = lo; e < hi; ++e) {
    const unsigned long long q = qfix(prob(srow[ckey_idx(lkey[e])], m), a.qscale);
    if ((double)(run + q) > Tq) { atomicMin(&S.jstar, e); break; }
    run += q;
  }
  __syncthreads();
  const int jstar = S.jstar;
  if (jstar < n && lo <= jstar && jstar < hi) {
    unsigned long long r = pbase;
    for (int e = lo; e < jstar; ++e) r += qfix(prob(srow[ckey_idx(lkey[e])], m), a.qscale);
    S.u64a = r;
    S.u64b = r + qfix(prob(srow[ckey_idx(lkey[jstar])], m), a.qscale);
  }
  __syncthreads();
  const bool ok = jstar < n && (double)S.u64a <= Tq - bq && (double)S.u64b > Tq + bq;
  const unsigned long long Kp = jstar < n ? lkey[jstar] : KEY_MAX;
  __syncthreads();
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
  __syncthreads();
  const int t = S.tok;
  __syncthreads();
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
    __syncthreads();
    if (threadIdx.x == 0) {
      const int lim = min(NT, V - base);
      for (int j = 0; j < lim; ++j) if (pv[j] != 0.0) sum = __dadd_rn(sum, pv[j]);
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) { S.dsum = __dmul_rn(u, sum); S.tok = (S.dsum == 0.0) ? 0 : -1; }
  __syncthreads();
  const double r = S.dsum;
  double acc = 0.0;
  for (int base = 0; base < V && S.tok < 0; base += NT) {
    const int i = base + threadIdx.x;
    double p = 0.0;
    if (i < V) { const float y = srow[i]; if (D(y, i)) p = prob(y, md); }
    pv[threadIdx.x] = p;
    __syncthreads();
    if (threadIdx.x == 0) {
      const int lim = min(NT, V - base);
      for (int j = 0; j < lim; ++j) {
        if (pv[j] == 0.0) continue;
        acc = __dadd_rn(acc, pv[j]);
        if (r <= acc) { S.tok = base + j; break; }
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0 && S.tok < 0) S.tok = V - 1;
  __syncthreads();
  const int t = S.tok;
  __syncthreads();
  return t;
}

// Draw over the index-sorted survivor list I[0..n); pv gets the probabilities.
__device__ int draw_list(const Args& a, const float* srow, const unsigned long long* I, int n, float md,
                         double u, double* pv, Shared& S) {
  for (int e = threadIdx.x; e < n; e += NT) pv[e] = prob(srow[(int)I[e]], md);
  __syncthreads();
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
  __syncthreads();
  unsigned long long run = base;
  for (int e = lo; e < hi; ++e) {
    const unsigned long long q = qfix(pv[e], a.qscale);
    if ((double)(run + q) >= rq) {
      atomicMin(&S.jstar, e);
      break;
    }
    run += q;
  }
  __syncthreads();
  const int js = S.jstar;
  if (js < n && lo <= js && js < hi) {
    unsigned long long r = base;
    for (int e = lo; e < js; ++e) r += qfix(pv[e], a.qscale);
    S.u64a = r;
    S.u64b = r + qfix(pv[js], a.qscale);
  }
  __syncthreads();
  const bool ok = SQ > 0 && js < n && (double)S.u64a < rq - bq && (double)S.u64b > rq + bq;
  __syncthreads();
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
  __syncthreads();
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
  __syncthreads();
  const int tok = S.tok;
  const bool ok = tok >= 0 && (double)S.u64a < rq - bq && (double)S.u64b > rq + bq;
  __syncthreads();
  if (ok) return tok;
  if (threadIdx.x == 0) atomicAdd(&a.counters[C4S_CNT_DRAW_EXACT_FALLBACK], 1ull);
  return draw_exact_row(srow, V, md, u, pv, S, D);
}

__global__ void __launch_bounds__(NT, 4) rows_kernel(Args a) {
  extern __shared__ __align__(16) unsigned char dsm[];
  __shared__ Shared S;
  const int V = a.V;
  const Layout L = layout_for(V);
  float* rowbuf = reinterpret_cast<float*>(dsm + L.row);
  unsigned* bitmap = reinterpret_cast<unsigned*>(dsm + L.bitmap);
  unsigned* cnt = reinterpret_cast<unsigned*>(dsm + L.cnt);
  unsigned long long* mass = reinterpret_cast<unsigned long long*>(dsm + L.mass);
  unsigned long long* lkey = reinterpret_cast<unsigned long long*>(dsm + L.key);
  double* pv = reinterpret_cast<double*>(dsm + L.pv);
  const int tid = threadIdx.x;

  if (tid == 0) mbar_init(&S.bar, 1);
  __syncthreads();
  unsigned phase = 0;

  for (int row = blockIdx.x; row < a.B; row += gridDim.x) {
    const c4s_row_params P = a.params[(long long)row * a.params_stride];
    if (a.mode == MODE_SAMPLE && a.active && !a.active[row]) {
      if (tid == 0) a.out_ids[row] = -1;
      continue;
    }
    const bool sample = a.mode == MODE_SAMPLE;
    const int st = sample ? (C4S_STAGE_PENALTY | C4S_STAGE_TEMPERATURE | C4S_STAGE_TOP_K | C4S_STAGE_TOP_P)
                          : (a.mode == MODE_PROCESS ? a.stages : 0);

    // ---- 1. stage the row --------------------------------------------------
    const float* g = (a.mode == MODE_PROCESS ? a.inout : a.logits) + (long long)row * a.ld;
    const unsigned long long ga = (unsigned long long)g;
    int head = (int)(((16u - (unsigned)(ga & 15ull)) & 15u) >> 2);
    if (head > V) head = V;
    const int body = ((V - head) >> 2) << 2;
    float* srow = rowbuf + ((4 - head) & 3);
    if (tid == 0 && body > 0) {
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&S.bar, (unsigned)body * 4u);
      bulk_g2s(srow + head, g + head, (unsigned)body * 4u, &S.bar);
    }
    for (int i = tid; i < head; i += NT) srow[i] = g[i];
    for (int i = head + body + tid; i < V; i += NT) srow[i] = g[i];

    const bool do_pen = (st & C4S_STAGE_PENALTY) && a.hist_off && P.repetition_penalty != 1.0f;
    long long h0 = 0, h1 = 0;
    if (do_pen) {
      h0 = a.hist_off[row];
      h1 = a.hist_off[row + 1];
      if (h0 < 0 || h1 < h0 || h1 > a.hist_total) {
        if (tid == 0) atomicOr(a.errflags, C4S_DEVERR_HIST_RANGE);
        h0 = h1 = 0;
      }
      for (int w = tid; w < (V + 31) / 32; w += NT) bitmap[w] = 0u;
    }
    int hid[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const long long j = h0 + tid + (long long)q * NT;
      hid[q] = (j < h1) ? a.hist[j] : -1;
    }
    if (tid == 0) {
      bool ok = true;
      if (body > 0) ok = mbar_wait_bounded(&S.bar, phase);
      S.abort_row = ok ? 0 : 1;
      if (!ok) atomicOr(a.errflags, C4S_DEVERR_TIMEOUT);
    }
    if (body > 0) phase ^= 1u;
    __syncthreads();
    if (S.abort_row) return;

    // ---- 2. repetition penalty ------------------------------------------------
    if (do_pen) {
      const float pen = P.repetition_penalty;
      auto apply = [&](int t) {
        if ((unsigned)t < (unsigned)V) {
          const unsigned bit = 1u << (t & 31);
          const unsigned old = atomicOr(&bitmap[t >> 5], bit);
          if (!(old & bit)) {
            const float s = srow[t];
            srow[t] = (s < 0.0f) ? __fmul_rn(s, pen) : __fdiv_rn(s, pen);
          }
        }
      };
#pragma unroll
      for (int q = 0; q < 8; ++q) apply(hid[q]);
      for (long long j = h0 + tid + 8LL * NT; j < h1; j += NT) apply(a.hist[j]);
      __syncthreads();
    }

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
      __syncthreads();
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
      __syncthreads();
      continue;
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
        __syncthreads();
        for (int i = tid; i < V; i += NT) {
          const int b = vbin(m, srow[i]);
          if (b < NBIN - 1) atomicAdd(&cnt[b], 1u);
        }
        __syncthreads();
        if (tid < 32)
          warp_find_bin<unsigned>([&](int j) { return cnt[j]; }, (unsigned)P.top_k, false, &S.c, &S.cbefore);
        __syncthreads();
        const int c = S.c;
        const int nle = (c < NBIN - 1) ? (int)(S.cbefore + cnt[c]) : LIST_CAP + 1;
        __syncthreads();
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
      __syncthreads();
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
        __syncthreads();
        const int np = next_pow2(max(nk, 1));
#pragma unroll
        for (int q = 0; q < LIST_CAP / NT; ++q) {
          const int e = tid + q * NT;
          if (e < np) lkey[e] = tmp[q];
        }
        __syncthreads();
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
    __syncthreads();
  }
}

__global__ void seed_kernel(unsigned long long* s, int B, unsigned long long seed, long long off) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) {
    const unsigned long long base = seed ? seed : 0x9E3779B97F4A7C15ull;
    s[b] = base + (unsigned long long)(off + b) * 0x100000001b3ull;
  }
}

}  // namespace c4s

// ============================================================================
// Host side: context and C ABI.
// ============================================================================
struct c4s_ctx {
  int device = 0;
  int max_vocab = 0;
  int num_sms = 0;
  int scratch_ctas = 0;
  int scratch_stride = 0;
  unsigned long long* d_scratch = nullptr;
  unsigned* d_err = nullptr;
  unsigned long long* d_counters = nullptr;
  c4s_row_params* d_default_params = nullptr;  // one zeroed struct (argmax reads no field)
  int debug = 0;
  int cached_V = -1;
  int cached_occ = 0;
  std::string last_error;
};

namespace {

int fail(c4s_ctx* ctx, int code, const std::string& msg) {
  if (ctx) ctx->last_error = msg;
  return code;
}

int cuda_fail(c4s_ctx* ctx, cudaError_t e, const char* what) {
  return fail(ctx, C4S_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Makes ctx->device current for the lifetime of the guard.
struct DeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) { ok = false; return; }
    if (prev != dev && cudaSetDevice(dev) != cudaSuccess) ok = false;
  }
  ~DeviceGuard() {
    int cur;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

int occupancy(c4s_ctx* ctx, int V, size_t smem) {
  if (ctx->cached_V == V) return ctx->cached_occ;
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, c4s::rows_kernel, c4s::NT, smem) != cudaSuccess)
    occ = 1;
  occ = std::max(1, occ);
  ctx->cached_V = V;
  ctx->cached_occ = occ;
  return occ;
}

int launch_rows(c4s_ctx* ctx, c4s::Args& a, void* stream) {
  using namespace c4s;
  if (a.B == 0) return C4S_OK;
  const size_t smem = layout_for(a.V).total;
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, C4S_ERR_CUDA, "cannot select the context's device");
  const int occ = occupancy(ctx, a.V, smem);
  const int grid = std::min<long long>((long long)a.B, (long long)std::min(occ, 8) * ctx->num_sms);
  if (grid > ctx->scratch_ctas) return fail(ctx, C4S_ERR_CAPACITY, "grid exceeds scratch slabs");
  a.scratch = ctx->d_scratch;
  a.scratch_stride = ctx->scratch_stride;
  a.errflags = ctx->d_err;
  a.counters = ctx->d_counters;
  a.debug = ctx->debug;
  int lg = 0;
  while ((1 << lg) < a.V) ++lg;
  a.qscale = std::ldexp(1.0, 62 - std::max(lg, 1));
  rows_kernel<<<grid, NT, smem, (cudaStream_t)stream>>>(a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(ctx, e, "rows_kernel launch");
  return C4S_OK;
}

int check_common(c4s_ctx* ctx, int B, int V, long long ld) {
  if (!ctx) return C4S_ERR_INVALID;
  if (B < 0) return fail(ctx, C4S_ERR_INVALID, "B < 0");
  if (V < 1) return fail(ctx, C4S_ERR_INVALID, "V < 1");
  if (V > ctx->max_vocab) return fail(ctx, C4S_ERR_CAPACITY, "V above the context's max_vocab");
  if (ld < V) return fail(ctx, C4S_ERR_INVALID, "ld < V");
  return C4S_OK;
}

}  // namespace

extern "C" {

int c4s_version(void) { return C4S_ABI_VERSION; }

const char* c4s_status_string(int s) {
  switch (s) {
    case C4S_OK: return "ok";
    case C4S_ERR_INVALID: return "invalid argument";
    case C4S_ERR_CUDA: return "CUDA error";
    case C4S_ERR_CAPACITY: return "capacity exceeded";
    case C4S_ERR_DEVICE: return "device-side error";
    case C4S_ERR_TIMEOUT: return "device wait timed out";
    case C4S_ERR_NCCL: return "collective failed";
    default: return "unknown status";
  }
}

int c4s_create(c4s_ctx** out, int32_t max_vocab, int32_t device) {
  if (!out) return C4S_ERR_INVALID;
  *out = nullptr;
  if (max_vocab < 1 || max_vocab > c4s::MAX_VOCAB || device < 0) return C4S_ERR_INVALID;
  c4s_ctx* ctx = new c4s_ctx();
  ctx->device = device;
  ctx->max_vocab = max_vocab;
  DeviceGuard dg(device);
  if (!dg.ok) { delete ctx; return C4S_ERR_CUDA; }
  cudaDeviceProp prop;
  cudaError_t e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) { delete ctx; return C4S_ERR_CUDA; }
  if (prop.major != 10) { delete ctx; return C4S_ERR_CUDA; }  // built for sm_100a only
  ctx->num_sms = prop.multiProcessorCount;
  // The attribute is per kernel (not per context): always allow the largest
  // row any context may launch, so contexts of different sizes coexist.
  const size_t smem_max = c4s::layout_for(c4s::MAX_VOCAB).total;
  e = cudaFuncSetAttribute(c4s::rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_max);
  if (e != cudaSuccess) { delete ctx; return C4S_ERR_CUDA; }
  int p2 = 1;
  while (p2 < max_vocab) p2 <<= 1;
  ctx->scratch_stride = p2;
  ctx->scratch_ctas = ctx->num_sms * 8;
  e = cudaMalloc(&ctx->d_scratch, (size_t)ctx->scratch_ctas * p2 * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMalloc(&ctx->d_err, sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMalloc(&ctx->d_counters, C4S_NUM_COUNTERS * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMalloc(&ctx->d_default_params, sizeof(c4s_row_params));
  if (e == cudaSuccess) e = cudaMemset(ctx->d_default_params, 0, sizeof(c4s_row_params));
  if (e == cudaSuccess) e = cudaMemset(ctx->d_err, 0, sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemset(ctx->d_counters, 0, C4S_NUM_COUNTERS * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(ctx->d_scratch); cudaFree(ctx->d_err); cudaFree(ctx->d_counters);
    cudaFree(ctx->d_default_params);
    delete ctx;
    return C4S_ERR_CUDA;
  }
  *out = ctx;
  return C4S_OK;
}

int c4s_destroy(c4s_ctx* ctx) {
  if (!ctx) return C4S_ERR_INVALID;
  {
    DeviceGuard dg(ctx->device);
    cudaFree(ctx->d_scratch);
    cudaFree(ctx->d_err);
    cudaFree(ctx->d_counters);
    cudaFree(ctx->d_default_params);
  }
  delete ctx;
  return C4S_OK;
}

const char* c4s_last_error(const c4s_ctx* ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

int c4s_set_debug(c4s_ctx* ctx, int32_t flags) {
  if (!ctx) return C4S_ERR_INVALID;
  if (flags & ~(C4S_DEBUG_FORCE_EXACT | C4S_DEBUG_FORCE_BINS)) return fail(ctx, C4S_ERR_INVALID, "unknown debug flag");
  ctx->debug = flags;
  return C4S_OK;
}

int c4s_seed_states(uint64_t* d_state, int32_t B, uint64_t seed, int64_t row_offset, void* stream) {
  if (B < 0 || (B > 0 && !d_state)) return C4S_ERR_INVALID;
  if (B == 0) return C4S_OK;
  c4s::seed_kernel<<<(B + 255) / 256, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<unsigned long long*>(d_state), B, seed, row_offset);
  return cudaGetLastError() == cudaSuccess ? C4S_OK : C4S_ERR_CUDA;
}

int c4s_sample(c4s_ctx* ctx, const float* d_logits, int32_t B, int32_t V, int64_t ld, const int32_t* d_hist,
               const int64_t* d_hist_off, int64_t hist_total, const c4s_row_params* d_params,
               int32_t params_stride, uint64_t* d_rng, const uint8_t* d_active, int32_t* d_out_ids,
               float* d_out_logits, int64_t out_ld, void* stream) {
  int rc = check_common(ctx, B, V, ld);
  if (rc) return rc;
  if (B == 0) return C4S_OK;
  if (!d_logits || !d_params || !d_rng || !d_out_ids) return fail(ctx, C4S_ERR_INVALID, "null pointer");
  if (params_stride != 0 && params_stride != 1) return fail(ctx, C4S_ERR_INVALID, "params_stride not 0/1");
  if (d_hist_off && (!d_hist && hist_total > 0)) return fail(ctx, C4S_ERR_INVALID, "history ids missing");
  if (hist_total < 0) return fail(ctx, C4S_ERR_INVALID, "hist_total < 0");
  if (d_out_logits && out_ld < V) return fail(ctx, C4S_ERR_INVALID, "out_ld < V");
  if (((uintptr_t)d_logits & 3) || (d_out_logits && ((uintptr_t)d_out_logits & 3)))
    return fail(ctx, C4S_ERR_INVALID, "misaligned float pointer");
  c4s::Args a{};
  a.logits = d_logits;
  a.B = B; a.V = V; a.ld = ld;
  a.hist = d_hist; a.hist_off = reinterpret_cast<const long long*>(d_hist_off); a.hist_total = hist_total;
  a.params = d_params; a.params_stride = params_stride;
  a.rng = reinterpret_cast<unsigned long long*>(d_rng);
  a.active = d_active;
  a.out_ids = d_out_ids;
  a.out_logits = d_out_logits; a.out_ld = out_ld;
  a.mode = c4s::MODE_SAMPLE;
  return launch_rows(ctx, a, stream);
}

int c4s_process(c4s_ctx* ctx, float* d_logits, int32_t B, int32_t V, int64_t ld, const int32_t* d_hist,
                const int64_t* d_hist_off, int64_t hist_total, const c4s_row_params* d_params,
                int32_t params_stride, int32_t stages, void* stream) {
  int rc = check_common(ctx, B, V, ld);
  if (rc) return rc;
  if (B == 0) return C4S_OK;
  if (!d_logits || !d_params) return fail(ctx, C4S_ERR_INVALID, "null pointer");
  if (params_stride != 0 && params_stride != 1) return fail(ctx, C4S_ERR_INVALID, "params_stride not 0/1");
  if (stages & ~0xF) return fail(ctx, C4S_ERR_INVALID, "unknown stage bit");
  if (d_hist_off && (!d_hist && hist_total > 0)) return fail(ctx, C4S_ERR_INVALID, "history ids missing");
  if (hist_total < 0) return fail(ctx, C4S_ERR_INVALID, "hist_total < 0");
  if ((uintptr_t)d_logits & 3) return fail(ctx, C4S_ERR_INVALID, "misaligned float pointer");
  c4s::Args a{};
  a.inout = d_logits;
  a.B = B; a.V = V; a.ld = ld;
  a.hist = d_hist; a.hist_off = reinterpret_cast<const long long*>(d_hist_off); a.hist_total = hist_total;
  a.params = d_params; a.params_stride = params_stride;
  a.mode = c4s::MODE_PROCESS;
  a.stages = stages;
  return launch_rows(ctx, a, stream);
}

int c4s_argmax(c4s_ctx* ctx, const float* d_logits, int32_t B, int32_t V, int64_t ld, int32_t* d_out_ids,
               void* stream) {
  int rc = check_common(ctx, B, V, ld);
  if (rc) return rc;
  if (B == 0) return C4S_OK;
  if (!d_logits || !d_out_ids) return fail(ctx, C4S_ERR_INVALID, "null pointer");
  if ((uintptr_t)d_logits & 3) return fail(ctx, C4S_ERR_INVALID, "misaligned float pointer");
  c4s::Args a{};
  a.logits = d_logits;
  a.B = B; a.V = V; a.ld = ld;
  a.params = ctx->d_default_params;
  a.params_stride = 0;
  a.out_ids = d_out_ids;
  a.mode = c4s::MODE_ARGMAX;
  return launch_rows(ctx, a, stream);
}

int c4s_get_status(c4s_ctx* ctx, uint32_t* dev_errors, uint64_t* counters, int32_t reset, void* stream) {
  if (!ctx) return C4S_ERR_INVALID;
  DeviceGuard dg(ctx->device);
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "stream synchronize");
  unsigned err = 0;
  e = cudaMemcpy(&err, ctx->d_err, sizeof(unsigned), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "read error flags");
  if (counters) {
    e = cudaMemcpy(counters, ctx->d_counters, C4S_NUM_COUNTERS * sizeof(uint64_t), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "read counters");
  }
  if (dev_errors) *dev_errors = err;
  if (reset) {
    cudaMemset(ctx->d_err, 0, sizeof(unsigned));
    cudaMemset(ctx->d_counters, 0, C4S_NUM_COUNTERS * sizeof(unsigned long long));
    cudaDeviceSynchronize();
  }
  if (err & C4S_DEVERR_TIMEOUT) return fail(ctx, C4S_ERR_TIMEOUT, "a bulk-copy wait timed out");
  if (err) return fail(ctx, C4S_ERR_DEVICE, "history offsets out of range");
  return C4S_OK;
}

}  // extern "C"
