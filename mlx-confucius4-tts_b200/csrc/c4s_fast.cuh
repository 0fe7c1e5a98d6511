// c4s_fast.cuh -- the fast path of the fused sampling step (MODE_SAMPLE, rows
// of up to F_MAXV logits).
//
// A persistent CTA processes rows blockIdx.x, +gridDim.x, ... with the row in
// shared memory (4 CTAs per SM). The next row's logits are prefetched into
// L2 while the current one is processed, and its metadata (params, history
// window, xorshift state) arrives in shared memory by cp.async. Per row:
//   - repetition penalty: scatter over the history, de-duplicated with a
//     shared bitmap (sampling.cpp:19-28);
//   - one pass: row max, per-thread maxima, first index of the max;
//   - greedy rows: first index of the max (sampling.cpp:73-76);
//   - top-k (sampling.cpp:30-40): each warp takes the ceil(k/8)-th largest of
//     its 32 thread maxima and the least of these, tau, has at least k
//     elements above it; the candidates >= tau (a few k at most) are divided
//     by T and gathered without atomics; the k-th largest is then exact on
//     that list (x/T is monotone in x);
//   - top-p (sampling.cpp:42-71) and the draw (text2semantic.cpp:150-165):
//     with <= F_SORT survivors one warp sorts them, locates the crossings with
//     fixed-point prefix sums and accepts them outside a proven error band,
//     else repeats the reference's sequential double sums exactly. Larger
//     candidate lists use value bins (top-p) and index bins (the draw).
//   - rows without top-k: a float estimate (untempered-x reciprocal product,
//     __expf) locates the top-p crossing with per-thread private histograms
//     (no atomics) and then float bins over one coarse bin; the <= F_SORT
//     candidates of the crossing bin get exact values. Where the crossing is
//     inside the estimate's error band, an exact double pass over the row
//     decides; the draw likewise (index-order prefix, exact pass on demand).
// Rows outside the fast path's assumptions (all -inf, |logits/T| >= 2^18,
// min_tokens_to_keep > 1, top_k above 32 per full warp, an undecided double
// band) go through the general path in the same CTA, on the staged row.
#pragma once

#include "c4s_general.cuh"

namespace c4s {

constexpr int F_MAXV = 9212;             // widest row the fast kernel takes
constexpr int NB_Y = 256;                // value bins over candidate lists
constexpr float YBIN = 8.0f;             // width 1/8
constexpr int NB_I = 256;                // draw index bins (list path)
constexpr int F_SORT = 128;              // warp-sort capacity
constexpr int NB1 = 16;                  // rows without top-k: level-1 bins, width 2
constexpr float L1SCALE = 0.5f;
constexpr int NB2 = 256;                 // level-2 bins inside one level-1 bin
constexpr float L2SCALE = 128.0f;        // width 1/128
constexpr double EPS_F = 4.0e-5;         // relative error of the float estimates (with margin)

// Per-row metadata, fetched asynchronously one row ahead.
struct __align__(16) MetaSlot {
  c4s_row_params P;          // 24 B
  long long off0, off1;      // history window [off0, off1)
  unsigned long long rng;    // xorshift64 state before this step
  int active;
  int pad;
};

struct FastLayout {
  size_t row, bitmap, cnt, mass, un, ws, meta, total;
};
__host__ __device__ inline FastLayout fast_layout(int V) {
  FastLayout L;
  size_t o = 0;
  L.row = o;    o += align_up((size_t)(V + 8) * 4, 16);      // + float4 over-read of the last block
  L.bitmap = o; o += align_up((size_t)((V + 31) / 32) * 4, 16);
  L.cnt = o;    o += 256 * 4;
  L.mass = o;   o += 256 * 8;
  L.un = o;     o += (size_t)LIST_CAP * 16;     // lkey[1024] + pv[1024] | float[NB1][NT]
  L.ws = o;     o += F_SORT * 8;
  L.meta = o;   o += 2 * sizeof(MetaSlot);
  L.total = o;
  return L;
}
static_assert(LIST_CAP * 16 >= NB1 * NT * 4, "private histograms fit the union");
static_assert(NBIN == 256 && NB_Y == 256 && NB_I == 256, "bin arrays are 256 wide");

__device__ __forceinline__ int ybin(float m, float y) {
  float t = __fmul_rn(__fsub_rn(m, y), YBIN);
  t = fminf(t, (float)(NB_Y - 1));
  return (int)t;
}

__device__ __forceinline__ void prefetch_l2(const void* p, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  return v;
}

// Appends key to buf (capacity cap) for the lanes with pred; one shared
// atomic per warp. All lanes of the warp must call.
__device__ __forceinline__ void warp_append(bool pred, unsigned long long key, unsigned long long* buf, int cap,
                                            int* counter) {
  const unsigned bal = __ballot_sync(FULL, pred);
  if (bal == 0) return;
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(bal) - 1;
  int base = 0;
  if (lane == leader) base = atomicAdd(counter, __popc(bal));
  base = __shfl_sync(FULL, base, leader);
  if (pred) {
    const int pos = base + __popc(bal & ((1u << lane) - 1u));
    if (pos < cap) buf[pos] = key;
  }
}

struct SumD { __device__ double operator()(double a, double b) const { return a + b; } };
struct MinF { __device__ float operator()(float a, float b) const { return fminf(a, b); } };
struct MaxI { __device__ int operator()(int a, int b) const { return a > b ? a : b; } };

// Exclusive scan of one double per thread over the CTA; *total gets the sum.
__device__ __forceinline__ double block_exscan_f64(double v, double* red, double* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(FULL, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) red[warp] = x;
  __syncthreads();
  double wbase = 0.0, tot = 0.0;
#pragma unroll
  for (int w = 0; w < NWARP; ++w) {
    const double t = red[w];
    if (w < warp) wbase += t;
    tot += t;
  }
  __syncthreads();
  *total = tot;
  return wbase + x - v;
}

// Warp 0 search over NB bins (PER = NB/32 per lane), same contract as
// warp_find_bin: first logical bin whose inclusive running sum exceeds
// (strict) or reaches `target`.
template <int PER, typename T, typename Get>
__device__ __forceinline__ void warp_find_bin_n(Get get, T target, bool strict, int* c_out, T* before_out) {
  const int lane = threadIdx.x & 31;
  T loc[PER];
  T s = 0;
#pragma unroll
  for (int j = 0; j < PER; ++j) { loc[j] = get(lane * PER + j); s += loc[j]; }
  T incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T y = __shfl_up_sync(FULL, incl, o);
    if (lane >= o) incl += y;
  }
  const bool hit = strict ? (incl > target) : (incl >= target);
  const unsigned bal = __ballot_sync(FULL, hit);
  if (bal == 0) {
    const T tot = __shfl_sync(FULL, incl, 31);
    if (lane == 0) { *c_out = 32 * PER; *before_out = tot; }
    return;
  }
  const int L = __ffs(bal) - 1;
  if (lane == L) {
    T run = incl - s;
    int c = L * PER + PER - 1;
    T before = run;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const bool h = strict ? (run + loc[j] > target) : (run + loc[j] >= target);
      if (h) { c = L * PER + j; before = run; break; }
      run += loc[j];
    }
    *c_out = c;
    *before_out = before;
  }
}

// Exact top-p of the reference over ws[0..n) sorted ascending by ckey, by one
// warp: sequential double sum, per-term division, sequential cumulative sum.
// Returns the first position whose cumulative probability exceeds thr (n if
// none).
__device__ __forceinline__ int warp_topp_exact(const unsigned long long* ws, int n, float m, double thr,
                                               double* pv) {
  const int lane = threadIdx.x & 31;
  for (int e = lane; e < n; e += 32) pv[e] = prob(fkey_inv((unsigned)(ws[e] >> 32)), m);
  __syncwarp();
  double sum = 0.0;
  if (lane == 0)
    for (int e = 0; e < n; ++e) sum = __dadd_rn(sum, pv[e]);
  sum = __shfl_sync(FULL, sum, 0);
  for (int e = lane; e < n; e += 32) pv[e] = __ddiv_rn(pv[e], sum);
  __syncwarp();
  int js = n;
  if (lane == 0) {
    double cum = 0.0;
    for (int e = 0; e < n; ++e) {
      cum = __dadd_rn(cum, pv[e]);
      if (!(cum <= thr)) { js = e; break; }
    }
  }
  return __shfl_sync(FULL, js, 0);
}

// Exact draw of the reference over ws[0..n) sorted by index, keys
// (index << 32 | fkey(y)), by one warp. Returns the token.
__device__ __forceinline__ int warp_draw_exact(const unsigned long long* ws, int n, float md, double u, int V,
                                               double* pv) {
  const int lane = threadIdx.x & 31;
  for (int e = lane; e < n; e += 32) pv[e] = prob(fkey_inv((unsigned)ws[e]), md);
  __syncwarp();
  int tok = V - 1;
  if (lane == 0) {
    double sum = 0.0;
    for (int e = 0; e < n; ++e) sum = __dadd_rn(sum, pv[e]);
    const double r = __dmul_rn(u, sum);
    if (r == 0.0) {
      tok = 0;
    } else {
      double acc = 0.0;
      for (int e = 0; e < n; ++e) {
        acc = __dadd_rn(acc, pv[e]);
        if (r <= acc) { tok = (int)(ws[e] >> 32); break; }
      }
    }
  }
  return __shfl_sync(FULL, tok, 0);
}

// Warp-level inclusive prefix of fixed-point masses over ws[0..n) (blocked,
// 4 entries per lane, n <= 128); finds the first entry whose prefix
// (plus `before`) satisfies pred(prefix). Returns the entry (n if none) and
// the prefixes just before it and at it.
template <typename QOf, typename Pred>
__device__ __forceinline__ int warp_prefix_find(const unsigned long long* ws, int n, unsigned long long before,
                                                QOf qof, Pred pred, unsigned long long* prev_out,
                                                unsigned long long* cur_out) {
  const int lane = threadIdx.x & 31;
  unsigned long long q[4];
  unsigned long long s = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int e = lane * 4 + j;
    q[j] = e < n ? qof(ws[e]) : 0ull;
    s += q[j];
  }
  unsigned long long incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long y = __shfl_up_sync(FULL, incl, o);
    if (lane >= o) incl += y;
  }
  unsigned long long run = before + incl - s;
  int found = n;
  unsigned long long pv_ = 0, cv = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int e = lane * 4 + j;
    if (found == n && e < n && pred(run + q[j])) { found = e; pv_ = run; cv = run + q[j]; }
    run += q[j];
  }
  const unsigned bal = __ballot_sync(FULL, found < n);
  if (bal == 0) {
    *prev_out = __shfl_sync(FULL, run, 31);
    *cur_out = *prev_out;
    return n;
  }
  const int L = __ffs(bal) - 1;
  *prev_out = __shfl_sync(FULL, pv_, L);
  *cur_out = __shfl_sync(FULL, cv, L);
  return __shfl_sync(FULL, found, L);
}


// ---------------------------------------------------------------------------
// Small survivor set (ns <= F_SORT), one warp: ws[0..ns) holds the survivors
// of top-k as ckeys. Decides top-p and draws; each crossing is taken from
// fixed-point prefix sums when it lies outside the proven error band, else
// the reference's sequential sums are repeated exactly. exp() runs once per
// survivor. Returns the token; K* via *kstar. pv needs 2*F_SORT doubles.
// Whole warp must call.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int warp_small_row(unsigned long long* ws, int ns, bool presorted, float m, double thr,
                                              int mk, unsigned long long u53, double u, int V, double qs,
                                              double* pv, unsigned long long* kstar) {
  const int lane = threadIdx.x & 31;
  if (!presorted) warp_sort(ws, ns);
  else __syncwarp();
  unsigned long long q[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int e = lane * 4 + j;
    const double p = e < ns ? prob(fkey_inv((unsigned)(ws[e] >> 32)), m) : 0.0;
    if (e < ns) pv[e] = p;
    q[j] = qfix(p, qs);
  }
  __syncwarp();
  // blocked warp prefix: first entry whose inclusive prefix satisfies pred
  auto find = [&](const unsigned long long (&qq)[4], int n, auto pred, unsigned long long* prev,
                  unsigned long long* cur, unsigned long long* total) {
    const unsigned long long s = qq[0] + qq[1] + qq[2] + qq[3];
    unsigned long long incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long y = __shfl_up_sync(FULL, incl, o);
      if (lane >= o) incl += y;
    }
    *total = __shfl_sync(FULL, incl, 31);
    unsigned long long run = incl - s, pv_ = 0, cv = 0;
    int found = n;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = lane * 4 + j;
      if (found == n && e < n && pred(run + qq[j])) { found = e; pv_ = run; cv = run + qq[j]; }
      run += qq[j];
    }
    const unsigned bal = __ballot_sync(FULL, found < n);
    if (bal == 0) { *prev = *total; *cur = *total; return n; }
    const int L = __ffs(bal) - 1;
    *prev = __shfl_sync(FULL, pv_, L);
    *cur = __shfl_sync(FULL, cv, L);
    return __shfl_sync(FULL, found, L);
  };
  int js;
  if (thr < 0.0) {
    js = 0;                                             // p > 1: nothing removed
  } else if (thr == 0.0) {
    int first = ns;                                     // p == 1: only zero probabilities go
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = lane * 4 + j;
      if (e < ns && pv[e] > 0.0) first = e < first ? e : first;
    }
    js = (int)__reduce_min_sync(FULL, (unsigned)first);
  } else {
    unsigned long long prev, cur, SQ;
    const int e0 = find(q, ns, [&](unsigned long long A) { return false; }, &prev, &cur, &SQ);
    (void)e0;
    const double SQd = (double)SQ, Tq = __dmul_rn(thr, SQd), bq = band_q(ns, SQd);
    const int e = find(q, ns, [Tq](unsigned long long A) { return (double)A > Tq; }, &prev, &cur, &SQ);
    bool ok;
    if (mk >= 1 && e >= ns - 1) {
      // the last element is kept anyway: only the mass below it must be certain
      const unsigned long long below = (e == ns - 1) ? prev : SQ - qfix(pv[ns - 1], qs);
      ok = (double)below <= Tq - bq;
      js = ns - 1;
    } else {
      ok = (double)prev <= Tq - bq && (e == ns || (double)cur > Tq + bq);
      js = e;
    }
    if (!ok) js = warp_topp_exact(ws, ns, m, thr, pv + F_SORT);
  }
  const unsigned long long Kp = js < ns ? ws[js] : KEY_MAX;
  const unsigned long long Kk = mk <= 0 ? KEY_MAX : ws[ns - 1];
  const unsigned long long K = Kp < Kk ? Kp : Kk;
  *kstar = K;
  if (u53 == 0ull) return 0;
  int jf = 0;
  for (int e = lane; e < ns; e += 32) jf += (ws[e] < K) ? 1 : 0;
  jf = __reduce_add_sync(FULL, jf);
  const int nk = ns - jf;
  if (nk == 0) return 0;
  // survivors of top-p by index; the low word keeps their position in pv
  unsigned long long t[F_SORT / 32];
#pragma unroll
  for (int qq = 0; qq < F_SORT / 32; ++qq) {
    const int e = jf + lane + 32 * qq;
    t[qq] = e < ns ? (((unsigned long long)ckey_idx(ws[e]) << 32) | (unsigned)e) : KEY_MAX;
  }
  __syncwarp();
#pragma unroll
  for (int qq = 0; qq < F_SORT / 32; ++qq) {
    const int e = lane + 32 * qq;
    if (e < nk) ws[e] = t[qq];
  }
  __syncwarp();
  warp_sort(ws, nk);
  unsigned long long qd[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int e = lane * 4 + j;
    qd[j] = e < nk ? qfix(pv[(unsigned)ws[e]], qs) : 0ull;
  }
  unsigned long long prev, cur, S2;
  (void)find(qd, nk, [&](unsigned long long A) { return false; }, &prev, &cur, &S2);
  const double S2d = (double)S2, rq = __dmul_rn(u, S2d), bq2 = band_q(nk, S2d);
  const int e = find(qd, nk, [rq](unsigned long long A) { return (double)A >= rq; }, &prev, &cur, &S2);
  if (S2 > 0 && e < nk && (double)prev < rq - bq2 && (double)cur > rq + bq2) return (int)(ws[e] >> 32);
  // exact: the reference's sequential sums over the same probabilities, index order
  int tok = V - 1;
  if (lane == 0) {
    double sum = 0.0;
    for (int e2 = 0; e2 < nk; ++e2) sum = __dadd_rn(sum, pv[(unsigned)ws[e2]]);
    const double r = __dmul_rn(u, sum);
    if (r == 0.0) {
      tok = 0;
    } else {
      double acc = 0.0;
      for (int e2 = 0; e2 < nk; ++e2) {
        acc = __dadd_rn(acc, pv[(unsigned)ws[e2]]);
        if (r <= acc) { tok = (int)(ws[e2] >> 32); break; }
      }
    }
  }
  return __shfl_sync(FULL, tok, 0);
}

// ---------------------------------------------------------------------------
// Top-p and the draw over the survivors of top-k, lkey[0..ns) (unordered
// ckeys of the tempered values). Commits the id and the state and leaves K*
// in S.kp. Returns false to defer the row (nothing written then).
// ---------------------------------------------------------------------------
__device__ bool list_topp_draw(const Args& a, int row, int ns, float m_y, double thr, int mk,
                               unsigned long long u53, double u, unsigned long long xs, bool force_bins,
                               unsigned long long* lkey, double* pv, unsigned long long* ws,
                               unsigned long long* mass, Shared& S) {
  const int V = a.V;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  auto each = [&](auto&& f) {
    for (int e = tid; e < ns; e += NT) {
      const unsigned long long key = lkey[e];
      f(fkey_inv((unsigned)(key >> 32)), ckey_idx(key));
    }
  };
  if (ns <= F_SORT && !force_bins) {
    // one warp finishes the row
    if (warp == 0) {
      for (int e = lane; e < ns; e += 32) ws[e] = lkey[e];
      __syncwarp();
      unsigned long long K;
      const int t = warp_small_row(ws, ns, false, m_y, thr, mk, u53, u, V, a.qscale, pv, &K);
      if (lane == 0) {
        S.kp = K;
        a.out_ids[row] = t;
        a.rng[row] = xs;
      }
    }
    __syncthreads();
    return true;
  }
  // ---- top-p: fixed-point mass per value bin ----
  for (int j = tid; j < NB_Y; j += NT) mass[j] = 0ull;
  __syncthreads();
  unsigned long long kmax = 0, kminp = KEY_MAX;
  each([&](float y, int i) {
    const double pr = prob(y, m_y);
    atomicAdd(&mass[ybin(m_y, y)], qfix(pr, a.qscale));
    const unsigned long long key = ckey(y, i);
    kmax = key > kmax ? key : kmax;
    if (pr > 0.0) kminp = key < kminp ? key : kminp;
  });
  kmax = block_reduce(kmax, MaxU64(), S.red64);
  kminp = block_reduce(kminp, MinU64(), S.red64);
  const unsigned long long SQ = block_reduce(mass[tid], SumU64(), S.red64);
  const unsigned long long Kk = mk <= 0 ? KEY_MAX : kmax;
  const double SQd = (double)SQ, Tq = __dmul_rn(thr, SQd), bq = band_q(ns, SQd);
  unsigned long long Kp = 0ull;
  bool need_cross = true;
  if (thr < 0.0) {
    need_cross = false;                                   // p > 1: nothing removed
  } else if (thr == 0.0) {
    Kp = kminp;                                           // p == 1: only zero probabilities go
    need_cross = false;
  } else if (Tq >= SQd - a.qscale) {
    if ((mk >= 1 && SQd - a.qscale <= Tq - bq) || (mk <= 0 && SQd <= Tq - bq)) {
      Kp = KEY_MAX;                                       // crossing at the largest element at most
      need_cross = false;
    } else if (Tq >= SQd) {
      return false;
    }
  }
  if (need_cross) {
    const unsigned long long target = (unsigned long long)floor(Tq);
    if (warp == 0)
      warp_find_bin_n<NB_Y / 32, unsigned long long>([&](int j) { return mass[NB_Y - 1 - j]; }, target, true,
                                                     &S.c, &S.mbefore);
    if (tid == 0) S.slot = 0;
    __syncthreads();
    const int cb = NB_Y - 1 - S.c;
    each([&](float y, int i) {
      if (ybin(m_y, y) == cb) {
        const int sl = atomicAdd(&S.slot, 1);
        if (sl < F_SORT) ws[sl] = ckey(y, i);
      }
    });
    __syncthreads();
    const int nc = S.slot;
    if (nc > F_SORT) return false;
    if (warp == 0) {
      warp_sort(ws, nc);
      unsigned long long prev, cur;
      const double qs = a.qscale;
      const float my = m_y;
      const int e = warp_prefix_find(
          ws, nc, S.mbefore,
          [qs, my](unsigned long long key) { return qfix(prob(fkey_inv((unsigned)(key >> 32)), my), qs); },
          [Tq](unsigned long long A) { return (double)A > Tq; }, &prev, &cur);
      const bool ok = e < nc && (double)prev <= Tq - bq && (double)cur > Tq + bq;
      if (lane == 0) { S.defer = ok ? 0 : 1; S.kp = ok ? ws[e] : 0ull; }
    }
    __syncthreads();
    if (S.defer) return false;
    Kp = S.kp;
  }
  const unsigned long long ks = Kp < Kk ? Kp : Kk;
  if (tid == 0) atomicAdd(&a.counters[C4S_CNT_TOPP_BINNED], 1ull);

  // ---- draw over the survivors of top-p, in index order ----
  int tok = 0;
  if (u53 != 0ull) {
    int cl = 0;
    each([&](float y, int i) { cl += ckey(y, i) >= ks ? 1 : 0; });
    const int nk = block_reduce(cl, SumI(), S.redi);
    if (nk <= F_SORT && !force_bins) {
      if (tid == 0) S.slot = 0;
      __syncthreads();
      each([&](float y, int i) {
        if (ckey(y, i) >= ks) ws[atomicAdd(&S.slot, 1)] = ((unsigned long long)i << 32) | fkey(y);
      });
      __syncthreads();
      if (warp == 0) {
        warp_sort(ws, nk);
        const double qs = a.qscale;
        const float my = m_y;
        auto qd = [qs, my](unsigned long long key) { return qfix(prob(fkey_inv((unsigned)key), my), qs); };
        unsigned long long S2 = 0;
        for (int e = lane; e < nk; e += 32) S2 += qd(ws[e]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) S2 += __shfl_xor_sync(FULL, S2, o);
        const double S2d = (double)S2, rq = __dmul_rn(u, S2d), bq2 = band_q(nk, S2d);
        unsigned long long prev, cur;
        const int e = warp_prefix_find(ws, nk, 0ull, qd, [rq](unsigned long long A) { return (double)A >= rq; },
                                       &prev, &cur);
        int t;
        if (S2 > 0 && e < nk && (double)prev < rq - bq2 && (double)cur > rq + bq2) t = (int)(ws[e] >> 32);
        else t = nk == 0 ? 0 : warp_draw_exact(ws, nk, m_y, u, V, pv);
        if (lane == 0) S.tok = t;
      }
      __syncthreads();
      tok = S.tok;
    } else {
      for (int j = tid; j < NB_I; j += NT) mass[j] = 0ull;
      __syncthreads();
      const int ish = a.ishift;
      each([&](float y, int i) {
        if (ckey(y, i) >= ks) atomicAdd(&mass[i >> ish], qfix(prob(y, m_y), a.qscale));
      });
      __syncthreads();
      const unsigned long long SQ2 = block_reduce(mass[tid], SumU64(), S.red64);
      const double SQ2d = (double)SQ2, rq = __dmul_rn(u, SQ2d), bq2 = band_q(nk, SQ2d);
      const unsigned long long target = (unsigned long long)ceil(rq);
      if (warp == 0)
        warp_find_bin_n<NB_I / 32, unsigned long long>([&](int j) { return mass[j]; }, target, false, &S.c,
                                                       &S.mbefore);
      if (tid == 0) S.slot = 0;
      __syncthreads();
      const int ib = S.c;
      if (ib >= NB_I) return false;
      each([&](float y, int i) {
        if (ckey(y, i) >= ks && (i >> ish) == ib) ws[atomicAdd(&S.slot, 1)] = ((unsigned long long)i << 32) | fkey(y);
      });
      __syncthreads();
      const int nb = S.slot;
      if (warp == 0) {
        warp_sort(ws, nb);
        unsigned long long prev, cur;
        const double qs = a.qscale;
        const float my = m_y;
        const int e = warp_prefix_find(
            ws, nb, S.mbefore, [qs, my](unsigned long long key) { return qfix(prob(fkey_inv((unsigned)key), my), qs); },
            [rq](unsigned long long A) { return (double)A >= rq; }, &prev, &cur);
        const bool ok = SQ2 > 0 && e < nb && (double)prev < rq - bq2 && (double)cur > rq + bq2;
        if (lane == 0) { S.defer = ok ? 0 : 1; S.tok = ok ? (int)(ws[e] >> 32) : 0; }
      }
      __syncthreads();
      if (S.defer) return false;
      tok = S.tok;
      if (tid == 0) atomicAdd(&a.counters[C4S_CNT_DRAW_ROWPASS], 1ull);
    }
  }
  if (tid == 0) {
    a.out_ids[row] = tok;
    a.rng[row] = xs;
    S.kp = ks;
  }
  __syncthreads();
  return true;
}

// Warp-level exclusive/inclusive prefix over ws[0..n) (blocked, 4 per lane,
// n <= 128) of double values val(key), starting at `before`; finds the first
// entry whose inclusive prefix satisfies pred. Whole warp must call.
template <typename Val, typename Pred>
__device__ __forceinline__ int warp_prefix_find_d(const unsigned long long* ws, int n, double before, Val val,
                                                  Pred pred, double* prev_out, double* cur_out) {
  const int lane = threadIdx.x & 31;
  double q[4];
  double s = 0.0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int e = lane * 4 + j;
    q[j] = e < n ? val(ws[e]) : 0.0;
    s += q[j];
  }
  double incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(FULL, incl, o);
    if (lane >= o) incl += y;
  }
  double run = before + (incl - s);
  int found = n;
  double pv_ = 0.0, cv = 0.0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int e = lane * 4 + j;
    if (found == n && e < n && pred(run + q[j])) { found = e; pv_ = run; cv = run + q[j]; }
    run += q[j];
  }
  const unsigned bal = __ballot_sync(FULL, found < n);
  if (bal == 0) {
    *prev_out = __shfl_sync(FULL, run, 31);
    *cur_out = *prev_out;
    return n;
  }
  const int L = __ffs(bal) - 1;
  *prev_out = __shfl_sync(FULL, pv_, L);
  *cur_out = __shfl_sync(FULL, cv, L);
  return __shfl_sync(FULL, found, L);
}

// ---------------------------------------------------------------------------
// Row passes: thread t owns the 36 contiguous buffer positions [36t, 36t+36)
// (element index = position - shift), read as 9 aligned float4 (conflict-free
// in shared memory). f(x, i) is called in increasing i.
// ---------------------------------------------------------------------------
constexpr int OWN = 36;
static_assert(OWN * NT >= F_MAXV + 3, "the ownership blocks cover every row position");

template <typename F>
__device__ __forceinline__ void row_pass(const float* rowbuf, int shift, int V, F&& f) {
  const int p0 = threadIdx.x * OWN;
#pragma unroll
  for (int qq = 0; qq < OWN / 4; ++qq) {
    const int pos = p0 + 4 * qq;
    if (pos < V + shift) {
      const float4 v = *reinterpret_cast<const float4*>(rowbuf + pos);
      const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int i = pos + r - shift;
        if ((unsigned)i < (unsigned)V) f(vv[r], i);
      }
    }
  }
}

// fl(x / T) (IEEE float division, sampling.cpp:16) from the double product
// x * RN(1/T): its error is below one double ulp, so rounding it to float
// gives the correctly rounded quotient unless it lies within a few double
// ulps of a float rounding midpoint (or outside the normal range); those
// cases take the hardware division.
__device__ __forceinline__ float div_exact(float x, float T, double rTd) {
  const double q = __dmul_rn((double)x, rTd);
  const unsigned low = (unsigned)((unsigned long long)__double_as_longlong(q) & 0x1fffffffull);
  const double aq = fabs(q);
  if (!(aq >= 1.0e-30 && aq <= 1.0e30) || (low - 0x0ffffffcu) <= 8u) return __fdiv_rn(x, T);
  return __double2float_rn(q);
}

// Relative error bound of __expf(d) in units of 2^-23 (CUDA's documented
// maximum ulp error of __expf is 2 + floor(|1.16 d|)).
__device__ __forceinline__ float expf_ulps(float d) { return 2.0f + 1.16f * fabsf(d); }
constexpr double ULP_F = 1.1920928955078125e-07 * 1.02;   // 2^-23, with 2% margin

// ---------------------------------------------------------------------------
// One staged, penalised row through the fast path. Returns false to defer
// the row to the general path (nothing has been written for it then).
// ---------------------------------------------------------------------------
__device__ bool fast_row4(const Args& a, int row, const MetaSlot& M, const float* rowbuf, int shift, unsigned* cnt,
                          unsigned long long* mass, unsigned char* un, unsigned long long* ws, Shared& S) {
  const int V = a.V;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const c4s_row_params P = M.P;
  unsigned long long* lkey = reinterpret_cast<unsigned long long*>(un);
  double* pv = reinterpret_cast<double*>(un + LIST_CAP * 8);

  // ---- pass 1: row max, thread max, first index of the thread max --------------
  float tm = -INFINITY;
  int ti = 0x7fffffff;
  row_pass(rowbuf, shift, V, [&](float x, int i) {
    if (x > tm) { tm = x; ti = i; }
  });
  {
    const unsigned km = __reduce_max_sync(FULL, fkey(tm));
    if (lane == 0) S.redu[warp] = km;
  }
  if (tid == 0) { S.slot = 0; S.slot2 = 0; }
  __syncthreads();
  unsigned kall = S.redu[0];
#pragma unroll
  for (int w = 1; w < NWARP; ++w) kall = kall > S.redu[w] ? kall : S.redu[w];
  const float m_x = fkey_inv(kall);
  __syncthreads();

  // ---- greedy: first index of the max (all -inf: index 0) ----------------------
  if (P.greedy) {
    unsigned cand = (tm == m_x && ti != 0x7fffffff) ? (unsigned)ti : 0xffffffffu;
    cand = __reduce_min_sync(FULL, cand);
    if (lane == 0) S.redu[warp] = cand;
    __syncthreads();
    if (tid == 0) {
      unsigned b = S.redu[0];
      for (int w = 1; w < NWARP; ++w) b = S.redu[w] < b ? S.redu[w] : b;
      a.out_ids[row] = b == 0xffffffffu ? 0 : (int)b;
    }
    if (a.out_logits) {
      float* o = a.out_logits + (long long)row * a.out_ld;
      row_pass(rowbuf, shift, V, [&](float x, int i) { o[i] = x; });
    }
    return true;
  }

  // ---- sample rows: preconditions of the fast path --------------------------------
  const float T = P.temperature;
  const bool do_t = !(T == 1.0f || T <= 0.0f);
  if (!(m_x > -INFINITY && m_x < INFINITY)) return false;
  const float m_y = do_t ? __fdiv_rn(m_x, T) : m_x;
  if (!(fabsf(m_y) < 262144.0f)) return false;
  if (P.min_tokens_to_keep > 1) return false;
  if (a.debug & C4S_DEBUG_FORCE_EXACT) return false;
  const bool force_bins = (a.debug & C4S_DEBUG_FORCE_BINS) != 0;
  const int k = P.top_k;
  const bool do_k = k > 0 && k < V;
  // warps whose 32 lanes all own row positions: their thread maxima bound top-k
  const int wfull = min(NWARP, ((V + shift + OWN - 1) / OWN) >> 5);
  if (do_k && (wfull == 0 || k > wfull * 32)) return false;
  const double thr = __dsub_rn(1.0, (double)P.top_p);
  const int mk = P.min_tokens_to_keep;
  unsigned long long xs = M.rng;
  xs ^= xs << 13; xs ^= xs >> 7; xs ^= xs << 17;
  const unsigned long long u53 = xs >> 11;
  const double u = (double)u53 * 1.1102230246251565e-16;
  const double rTd = do_t ? 1.0 / (double)T : 1.0;
  auto yex = [&](float x) { return do_t ? div_exact(x, T, rTd) : x; };   // sampling.cpp:16

  float thresh_y = -INFINITY;
  if (do_k) {
    // ---- top-k: threshold from the thread maxima, candidates gathered ------------
    // Each full warp has >= kw thread maxima >= its kw-th largest, so at least
    // wfull*kw >= k elements are >= tau, the least of those over the full warps.
    const int kw = (k + wfull - 1) / wfull;
    unsigned key = fkey(tm);
#pragma unroll
    for (int kk = 2; kk <= 32; kk <<= 1) {
#pragma unroll
      for (int jj = kk >> 1; jj > 0; jj >>= 1) {
        const unsigned o = __shfl_xor_sync(FULL, key, jj);
        const bool keep_min = (((lane & jj) == 0) == ((lane & kk) == 0));
        key = keep_min ? (o < key ? o : key) : (o > key ? o : key);
      }
    }
    const unsigned wthr = __shfl_sync(FULL, key, 32 - kw);      // ascending: kw-th largest
    if (lane == 0) S.redu[warp] = wthr;
    __syncthreads();
    unsigned tkey = S.redu[0];
    for (int w = 1; w < wfull; ++w) tkey = S.redu[w] < tkey ? S.redu[w] : tkey;
    const float tau = fkey_inv(tkey);
    const float tau_lo = tau - (fabsf(tau) + 1.0f) * 3.814697265625e-06f;   // below tau by 2^-18 relative
    int cnt_t = 0;
    row_pass(rowbuf, shift, V, [&](float x, int) { cnt_t += x >= tau_lo ? 1 : 0; });
    int ng;
    int wpos = block_exscan_i32(cnt_t, S.redi, &ng);
    if (ng > LIST_CAP) return false;
    row_pass(rowbuf, shift, V, [&](float x, int i) {
      if (x >= tau_lo) lkey[wpos++] = ckey(yex(x), i);
    });
    __syncthreads();
    int ns;
    if (ng <= F_SORT) {
      if (warp == 0) {
        for (int e = lane; e < ng; e += 32) ws[e] = lkey[e];
        __syncwarp();
        warp_sort(ws, ng);
        const unsigned tk2 = (unsigned)(ws[ng - k] >> 32);
        int below = 0;
        for (int e = lane; e < ng; e += 32) below += ((unsigned)(ws[e] >> 32) < tk2) ? 1 : 0;
        below = __reduce_add_sync(FULL, below);
        const int nsv = ng - below;
        unsigned long long t4[F_SORT / 32];
#pragma unroll
        for (int q = 0; q < F_SORT / 32; ++q) {
          const int e = below + lane + 32 * q;
          t4[q] = e < ng ? ws[e] : KEY_MAX;
        }
        __syncwarp();
#pragma unroll
        for (int q = 0; q < F_SORT / 32; ++q) {
          const int e = lane + 32 * q;
          if (e < nsv) { ws[e] = t4[q]; lkey[e] = t4[q]; }
        }
        __syncwarp();
        int done = 0;
        if (!force_bins) {
          unsigned long long K;
          const int t = warp_small_row(ws, nsv, true, m_y, thr, mk, u53, u, V, a.qscale, pv, &K);
          if (lane == 0) { S.kp = K; a.out_ids[row] = t; a.rng[row] = xs; }
          done = 1;
        }
        if (lane == 0) { S.thresh_key = tk2; S.ns = nsv; S.done = done; }
      }
      __syncthreads();
      thresh_y = fkey_inv(S.thresh_key);
      ns = S.ns;
      if (!S.done && !list_topp_draw(a, row, ns, m_y, thr, mk, u53, u, xs, force_bins, lkey, pv, ws, mass, S))
        return false;
    } else {
      // count the candidates per value bin, sort the bin of the k-th largest
      for (int jb = tid; jb < NB_Y; jb += NT) cnt[jb] = 0u;
      __syncthreads();
      for (int e = tid; e < ng; e += NT) atomicAdd(&cnt[ybin(m_y, fkey_inv((unsigned)(lkey[e] >> 32)))], 1u);
      __syncthreads();
      if (warp == 0)
        warp_find_bin_n<NB_Y / 32, unsigned>([&](int jb) { return cnt[jb]; }, (unsigned)k, false, &S.c,
                                             &S.cbefore);
      if (tid == 0) S.slot = 0;
      __syncthreads();
      const int cb = S.c;
      if (cb >= NB_Y) return false;
      const int nb = (int)cnt[cb];
      if (nb > F_SORT) return false;
      for (int e = tid; e < ng; e += NT) {
        const unsigned long long kk2 = lkey[e];
        if (ybin(m_y, fkey_inv((unsigned)(kk2 >> 32))) == cb) ws[atomicAdd(&S.slot, 1)] = kk2;
      }
      __syncthreads();
      if (warp == 0) {
        warp_sort(ws, nb);
        const int kk = k - (int)S.cbefore;                 // 1 <= kk <= nb
        if (lane == 0) S.thresh_key = (unsigned)(ws[nb - kk] >> 32);
      }
      __syncthreads();
      const unsigned tk2 = S.thresh_key;
      unsigned long long mine[LIST_CAP / NT];
      int c2 = 0;
#pragma unroll
      for (int q = 0; q < LIST_CAP / NT; ++q) {
        const int e = tid + q * NT;
        mine[q] = (e < ng && (unsigned)(lkey[e] >> 32) >= tk2) ? lkey[e] : KEY_MAX;
        c2 += mine[q] != KEY_MAX ? 1 : 0;
      }
      int nsv;
      int wp = block_exscan_i32(c2, S.redi, &nsv);     // its barriers order the reads before the writes
#pragma unroll
      for (int q = 0; q < LIST_CAP / NT; ++q)
        if (mine[q] != KEY_MAX) lkey[wp++] = mine[q];
      __syncthreads();
      thresh_y = fkey_inv(tk2);
      ns = nsv;
      if (!list_topp_draw(a, row, ns, m_y, thr, mk, u53, u, xs, force_bins, lkey, pv, ws, mass, S)) return false;
    }
  } else {
    // ---- no top-k: float estimates of exact values --------------------------------
    auto coarse = [&](float d) { return min(NB1 - 1, (int)(fmaxf(-d, 0.0f) * L1SCALE)); };
    auto fine = [&](float d, float lo1) { return min(NB2 - 1, max(0, (int)((-d - lo1) * L2SCALE))); };
    float* H = reinterpret_cast<float*>(un);
#pragma unroll
    for (int b = 0; b < NB1; ++b) H[b * NT + tid] = 0.0f;
    double st = 0.0, eb = 0.0;
    float dmin = 0.0f;
    int nf = 0, kim = -1;
    row_pass(rowbuf, shift, V, [&](float x, int i) {
      if (x > -INFINITY) {
        const float y = yex(x);
        const float d = __fsub_rn(y, m_y);
        const float p = __expf(d);
        st += p;
        eb += expf_ulps(d) * p;
        ++nf;
        dmin = fminf(dmin, d);
        H[coarse(d) * NT + tid] += p;
        if (y == m_y) kim = i;
      }
    });
    const int nfa = block_reduce(nf, SumI(), S.redi);
    if (nfa <= F_SORT && !force_bins) {
      // few finite logits: exact list in index order
      int cf = nf;
      int wpos = block_exscan_i32(cf, S.redi, &cf);
      row_pass(rowbuf, shift, V, [&](float x, int i) {
        if (x > -INFINITY) lkey[wpos++] = ckey(yex(x), i);
      });
      __syncthreads();
      if (!list_topp_draw(a, row, nfa, m_y, thr, mk, u53, u, xs, false, lkey, pv, ws, mass, S)) return false;
    } else {
      const int kima = block_reduce(kim, MaxI(), S.redi);
      const double Sh = block_reduce(st, SumD(), S.redd);
      const double Eh = block_reduce(eb, SumD(), S.redd) * ULP_F + 1e-30 * nfa;
      const float dmn = block_reduce(dmin, MinF(), S.redf);
      for (int bb = warp; bb < NB1; bb += NWARP) {
        float v = 0.0f;
#pragma unroll
        for (int q = 0; q < NT / 32; ++q) v += H[bb * NT + lane + 32 * q];
        v = warp_sum_f(v);
        if (lane == 0) S.l1[bb] = v;
      }
      __syncthreads();
      const unsigned long long Kk = mk <= 0 ? KEY_MAX : ckey(m_y, kima);
      unsigned long long Kp = 0ull;
      int status = 0;                                     // 0 decided, 1 exact pass, 2 defer
      int nc = 0;
      // estimate error: each prefix and the total are within Eh of the exact
      // sums of the same terms; the reference's own rounding adds ~n ulps
      const double Th = thr * Sh;
      const double band = 2.0 * Eh + 2.0 * (4.0 * nfa + 16.0) * U53 * Sh;
      if (thr < 0.0) {
        Kp = 0ull;                                        // p > 1: nothing removed
      } else if (thr == 0.0) {
        if (dmn > -700.0f) Kp = 0ull;                     // p == 1: no exp() can underflow to 0
        else status = 2;
      } else {
        int c1 = -1;
        double cum = 0.0;
        for (int b = NB1 - 1; b >= 0; --b) {
          if (cum + (double)S.l1[b] > Th) { c1 = b; break; }
          cum += (double)S.l1[b];
        }
        if (c1 < 0) {
          if (mk >= 1 && Sh - 1.0 <= Th - band) Kp = KEY_MAX;   // only the kept maximum survives
          else status = 2;
        } else if (c1 == NB1 - 1) {
          status = 2;                                     // crossing in the far tail
        } else {
          // level 2: float bins inside the coarse bin (localisation only)
          float* L2p = reinterpret_cast<float*>(cnt);
          unsigned* L2n = reinterpret_cast<unsigned*>(mass);
          for (int jb = tid; jb < NB2; jb += NT) { L2p[jb] = 0.0f; L2n[jb] = 0u; }
          __syncthreads();
          const float lo1 = 2.0f * (float)c1;
          row_pass(rowbuf, shift, V, [&](float x, int) {
            if (x > -INFINITY) {
              const float d = __fsub_rn(yex(x), m_y);
              if (coarse(d) == c1) {
                const int f = fine(d, lo1);
                atomicAdd(&L2p[f], __expf(d));
                atomicAdd(&L2n[f], 1u);
              }
            }
          });
          __syncthreads();
          if (warp == 0)
            warp_find_bin_n<NB2 / 32, float>([&](int jb) { return L2p[NB2 - 1 - jb]; }, (float)(Th - cum),
                                             true, &S.c, &S.fbefore);
          __syncthreads();
          const int jc = S.c;
          if (jc >= NB2 || (int)L2n[NB2 - 1 - jc] > F_SORT) {
            status = 2;
          } else {
            const int c2 = NB2 - 1 - jc;
            // the crossing bin's elements (exact keys) and the estimated mass below it
            double bl = 0.0;
            row_pass(rowbuf, shift, V, [&](float x, int i) {
              if (x > -INFINITY) {
                const float y = yex(x);
                const float d = __fsub_rn(y, m_y);
                const int cb1 = coarse(d);
                if (cb1 > c1) {
                  bl += __expf(d);
                } else if (cb1 == c1) {
                  const int f = fine(d, lo1);
                  if (f > c2) bl += __expf(d);
                  else if (f == c2) {
                    const int sl = atomicAdd(&S.slot2, 1);
                    if (sl < F_SORT) ws[sl] = ckey(y, i);
                  }
                }
              }
            });
            const double before = block_reduce(bl, SumD(), S.redd);
            nc = min(S.slot2, F_SORT);
            if (warp == 0) {
              warp_sort(ws, nc);
              const float my = m_y;
              double prev, cur;
              const int e = warp_prefix_find_d(
                  ws, nc, before, [my](unsigned long long kq) { return prob(fkey_inv((unsigned)(kq >> 32)), my); },
                  [Th](double A) { return A > Th; }, &prev, &cur);
              const bool ok = e < nc && prev <= Th - band && cur > Th + band;
              if (lane == 0) { S.kp = ok ? ws[e] : 0ull; S.defer = ok ? 0 : 1; }
            }
            __syncthreads();
            if (S.defer) status = 1;
            else Kp = S.kp;
          }
        }
      }
      if (status == 1) {
        // exact double sums over the row decide among the candidates
        const unsigned long long klo = ws[0];
        double se = 0.0, be = 0.0;
        row_pass(rowbuf, shift, V, [&](float x, int i) {
          if (x > -INFINITY) {
            const float y = yex(x);
            const double p = prob(y, m_y);
            se += p;
            if (ckey(y, i) < klo) be += p;
          }
        });
        se = block_reduce(se, SumD(), S.redd);
        be = block_reduce(be, SumD(), S.redd);
        if (warp == 0) {
          const float my = m_y;
          const double Te = thr * se, bqe = 2.0 * ((4.0 * nfa + 16.0) * U53 * se);
          double prev, cur;
          const int e = warp_prefix_find_d(
              ws, nc, be, [my](unsigned long long kq) { return prob(fkey_inv((unsigned)(kq >> 32)), my); },
              [Te](double A) { return A > Te; }, &prev, &cur);
          const bool ok = e < nc && prev <= Te - bqe && cur > Te + bqe;
          if (lane == 0) { S.kp = ok ? ws[e] : 0ull; S.defer = ok ? 0 : 1; }
        }
        __syncthreads();
        if (S.defer) return false;
        Kp = S.kp;
        if (tid == 0) atomicAdd(&a.counters[C4S_CNT_TOPP_EXACT_FALLBACK], 1ull);
      } else if (status == 2) {
        return false;
      }
      const unsigned long long ks = Kp < Kk ? Kp : Kk;
      if (tid == 0) atomicAdd(&a.counters[C4S_CNT_TOPP_BINNED], 1ull);

      // ---- draw: index-order prefix of the estimates, exact pass on demand ----
      int tok = 0;
      if (u53 != 0ull && ks != KEY_MAX) {
        for (int pass = 0; pass < 2; ++pass) {
          const bool exact = pass == 1;
          double loc = 0.0, el = 0.0;
          int nl = 0;
          row_pass(rowbuf, shift, V, [&](float x, int i) {
            if (x > -INFINITY) {
              const float y = yex(x);
              if (ckey(y, i) >= ks) {
                const float d = __fsub_rn(y, m_y);
                if (exact) {
                  loc += prob(y, m_y);
                } else {
                  const float p = __expf(d);
                  loc += p;
                  el += expf_ulps(d) * p;
                }
                ++nl;
              }
            }
          });
          if (tid == 0) S.tok = -1;
          double Sk;
          const double base = block_exscan_f64(loc, S.redd, &Sk);
          const int nk = block_reduce(nl, SumI(), S.redi);
          const double Ek = exact ? 0.0 : block_reduce(el, SumD(), S.redd) * ULP_F;
          const double rq = u * Sk;
          const double bd = 2.0 * Ek + 2.0 * (4.0 * nk + 16.0) * U53 * Sk;
          if (Sk > 0.0 && base < rq && base + loc >= rq) {
            double run = base;
            int found = -1;
            double fprev = 0.0, fcur = 0.0;
            row_pass(rowbuf, shift, V, [&](float x, int i) {
              if (found < 0 && x > -INFINITY) {
                const float y = yex(x);
                if (ckey(y, i) >= ks) {
                  const double p = exact ? prob(y, m_y) : (double)__expf(__fsub_rn(y, m_y));
                  if (run + p >= rq) { found = i; fprev = run; fcur = run + p; }
                  run += p;
                }
              }
            });
            if (found >= 0) { S.tok = found; S.d1 = fprev; S.d2 = fcur; }
          }
          __syncthreads();
          const bool ok = (Sk == 0.0) || (S.tok >= 0 && S.d1 < rq - bd && S.d2 > rq + bd);
          const int t = (Sk == 0.0) ? 0 : S.tok;
          __syncthreads();
          if (ok) { tok = t; break; }
          if (exact) return false;
          if (tid == 0) atomicAdd(&a.counters[C4S_CNT_DRAW_EXACT_FALLBACK], 1ull);
        }
      }
      if (tid == 0) {
        a.out_ids[row] = tok;
        a.rng[row] = xs;
        S.kp = ks;
      }
      __syncthreads();
    }
  }

  // ---- processed logits (on request) ------------------------------------------------
  if (a.out_logits) {
    const unsigned long long kst = S.kp;
    float* o = a.out_logits + (long long)row * a.out_ld;
    row_pass(rowbuf, shift, V, [&](float x, int i) {
      const float y = yex(x);
      const bool masked = (y < thresh_y) || (y > -INFINITY && ckey(y, i) < kst);
      o[i] = masked ? -INFINITY : y;
    });
  }
  return true;
}

// ---------------------------------------------------------------------------
// The fast kernel: rows blockIdx.x, +gridDim.x, ...; metadata of the next
// row by cp.async and its logits prefetched into L2 while the current row is
// processed. Rows the fast path declines take the general path in place.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NT, 4) fast_kernel(Args a) {
  extern __shared__ __align__(16) unsigned char dsm[];
  __shared__ Shared S;
  const int V = a.V;
  const FastLayout L = fast_layout(V);
  float* rowbuf = reinterpret_cast<float*>(dsm + L.row);
  unsigned* bitmap = reinterpret_cast<unsigned*>(dsm + L.bitmap);
  unsigned* cnt = reinterpret_cast<unsigned*>(dsm + L.cnt);
  unsigned long long* mass = reinterpret_cast<unsigned long long*>(dsm + L.mass);
  unsigned char* un = dsm + L.un;
  unsigned long long* lkey = reinterpret_cast<unsigned long long*>(un);
  double* pv = reinterpret_cast<double*>(un + LIST_CAP * 8);
  unsigned long long* ws = reinterpret_cast<unsigned long long*>(dsm + L.ws);
  MetaSlot* meta = reinterpret_cast<MetaSlot*>(dsm + L.meta);
  const int tid = threadIdx.x;
  const int G = gridDim.x;
  const int nbitmap = (V + 31) / 32;

  if (tid == 0) mbar_init(&S.bar, 1);
  unsigned phase = 0;
  bool aborted = false;

  int act_pend = 1;
  auto issue_meta = [&](int r, MetaSlot& ms) {
    if (r >= a.B) return;
    const char* pp = reinterpret_cast<const char*>(a.params + (long long)r * a.params_stride);
    if (tid < 3) cp_async8(reinterpret_cast<char*>(&ms.P) + 8 * tid, pp + 8 * tid);
    else if (tid == 3) { if (a.hist_off) cp_async8(&ms.off0, a.hist_off + r); else ms.off0 = 0; }
    else if (tid == 4) { if (a.hist_off) cp_async8(&ms.off1, a.hist_off + r + 1); else ms.off1 = 0; }
    else if (tid == 5) cp_async8(&ms.rng, a.rng + r);
    else if (tid == 6) act_pend = a.active ? (int)a.active[r] : 1;
  };

  const int r0 = blockIdx.x;
  issue_meta(r0, meta[0]);
  cp_async_commit();
  if (tid == 6 && r0 < a.B) meta[0].active = act_pend;
  cp_async_wait<0>();
  __syncthreads();

  int j = 0;
  for (int row = r0; row < a.B; row += G, ++j) {
    MetaSlot& cur = meta[j & 1];
    MetaSlot& nxt = meta[(j + 1) & 1];
    const int next = row + G;
    issue_meta(next, nxt);
    cp_async_commit();
    if (cur.active) {
      const c4s_row_params P = cur.P;
      const Stage sg = stage_issue(a.logits + (long long)row * a.ld, V, rowbuf, &S.bar);
      if (tid == 0 && next < a.B) {
        // warm L2 with the next row while this one is processed
        const float* gn = a.logits + (long long)next * a.ld;
        const unsigned long long gna = (unsigned long long)gn;
        int hn = (int)(((16u - (unsigned)(gna & 15ull)) & 15u) >> 2);
        if (hn > V) hn = V;
        const int bn = ((V - hn) >> 2) << 2;
        if (bn > 0) prefetch_l2(gn + hn, (unsigned)bn * 4u);
      }
      const bool pen = a.hist_off && P.repetition_penalty != 1.0f;
      long long h0 = 0, h1 = 0;
      if (pen) {
        h0 = cur.off0;
        h1 = cur.off1;
        if (h0 < 0 || h1 < h0 || h1 > a.hist_total) {
          if (tid == 0) atomicOr(a.errflags, C4S_DEVERR_HIST_RANGE);
          h0 = h1 = 0;
        }
        for (int w = tid; w < nbitmap; w += NT) bitmap[w] = 0u;
      }
      int hid[8];
      hist_prefetch(a, h0, h1, hid);
      if (!stage_wait(a, sg, &S.bar, phase, S)) { aborted = true; break; }
      float* srow = rowbuf + sg.shift;
      if (pen) penalty_apply(a, srow, V, bitmap, P.repetition_penalty, hid, h0, h1);
      if (!fast_row4(a, row, cur, rowbuf, sg.shift, cnt, mass, un, ws, S)) {
        // outside the fast path's assumptions: the general path, same CTA, same staged row
        __syncthreads();
        if (tid == 0) atomicAdd(&a.counters[C4S_CNT_DEFERRED], 1ull);
        finish_general(a, row, P, C4S_STAGE_PENALTY | C4S_STAGE_TEMPERATURE | C4S_STAGE_TOP_K | C4S_STAGE_TOP_P,
                       srow, cnt, mass, lkey, pv, S);
      }
    } else if (tid == 0) {
      a.out_ids[row] = -1;
    }
    if (tid == 6 && next < a.B) nxt.active = act_pend;
    cp_async_wait<0>();
    __syncthreads();                                       // next metadata visible, buffers free
  }
  cp_async_wait<0>();
  if (aborted && tid == 0) mbar_wait_bounded(&S.bar, phase);   // let a timed-out copy drain (bounded)
}

}  // namespace c4s
