// c4s_fast.cuh -- the fast path of the fused sampling step (MODE_SAMPLE, rows
// of up to F_MAXV logits): three kernels per chunk of at most K_CHUNK rows.
//
//   row_kernel (persistent, NT threads, four CTAs per SM): thread t holds the
//     36 row elements of positions [36t, 36t+36) in registers, loaded with
//     16-byte streaming loads (no shared-memory row buffer, so many rows are
//     in flight per SM). It applies the repetition penalty through a
//     shared-memory bitmap of the row's history (sampling.cpp:19-28) and makes
//     every pass over the row from registers:
//       greedy rows: first index of the maximum (sampling.cpp:73-76);
//       top-k rows: each full warp takes the ceil(k/wfull)-th largest of its
//         lanes' maxima (of the two largest per lane when k > 64) and tau is
//         the least of those, so at least k elements are >= tau; the
//         candidates >= tau (minus a margin covering values that the
//         temperature division merges) form the row's list: top_k keeps
//         y >= (k-th largest y) and y = x/T is monotone, so every survivor is
//         in it (sampling.cpp:30-40);
//       rows without top-k: an octave histogram of error-bounded estimates
//         of the probabilities locates the top-p crossing; the octaves down
//         to it form the list, the deeper ones an estimated tail with a
//         proven bound. When that list would be too long the row kernel
//         finishes the row itself (sub-bins of the crossing octave, an exact
//         sort of one sub-bin, the draw over per-thread survivor masses).
//     Lists go to global memory (they stay in L2) with a per-row job record.
//   list_kernel (one warp per row): exact top-k threshold by bisection on the
//     value keys, exact double-precision probabilities, the top-p crossing
//     and the draw (sampling.cpp:42-71, text2semantic.cpp:150-165).
//   defer_kernel: the general path for the rare rows the others hand back
//     (non-finite maxima, |max/T| >= 2^18, min_tokens_to_keep != 1, lists
//     over LCAP, undecidable error bands).
//   mask_kernel (only when processed logits are requested): applies the
//     list kernel's top-k/top-p decisions to the tempered logits.
//
// Exactness: every decision taken from rounded or estimated sums is accepted
// only outside a proven error band; inside it the reference's sequential
// double sums are repeated exactly (or the row goes to the general path).
#pragma once

#include "c4s_general.cuh"

namespace c4s {

constexpr int F_MAXV = 9212;              // widest row the fast path takes
constexpr int OWN = 36;                   // row positions per row-kernel thread
constexpr int LCAP = 2048;                // candidates per list
constexpr int K_CHUNK = 4096;             // rows per launch sequence (list storage)
constexpr int NOCT = 30;                  // octaves of the estimate (<= 31: one warp lane each); bin NOCT = the rest
constexpr int BIG_SORT = 128;             // crossing sub-bin capacity (one warp sort)
constexpr int CAND_CAP = 2048;            // crossing-octave candidates
constexpr int LIST_WARPS = 8;             // list kernel: rows (warps) per CTA
static_assert(OWN * NT >= F_MAXV + 3, "the ownership blocks cover every row position");
static_assert(OWN <= 64, "per-thread candidate masks are 64 bits");

enum { JOB_NONE = 0, JOB_TOPK = 1, JOB_K0 = 2, JOB_DEFER = 3 };
enum { RES_DONE = 0, RES_DEFER = 1, RES_REFINE = 2 };

// Per-row job record: written by the row kernel, finished by the list kernel.
struct __align__(16) RowJob {
  int kind, n, k, status;
  float m_y;                 // row maximum after temperature
  unsigned ykex;             // JOB_K0: key of the largest value below the list (0: none)
  unsigned thresh_key;       // result: top-k threshold key (0: none)
  int pad;
  double thr, u;             // 1 - top_p; uniform of the draw
  double tail, tail_err;     // JOB_K0: estimated mass below the list and its error bound
  unsigned long long u53, xs;
  unsigned long long kstar;  // result: keys below K* are removed by top-p
  unsigned long long pad2;
};

// Per-row metadata, fetched asynchronously one row ahead.
struct __align__(16) MetaSlot {
  c4s_row_params P;          // 24 B
  long long off0, off1;      // history window [off0, off1)
  unsigned long long rng;    // xorshift64 state before this step
  int active;
  int pad;
};

// Dynamic shared memory of the row kernel: the staged row; for rows without
// top-k, after it is in registers, their octave columns and then the scratch
// of their big path (same area).
constexpr size_t RWORK_BYTES = (size_t)(NOCT + 1) * NT * 4;
// Every thread reads its whole ownership block (NT * OWN positions), so the
// buffer covers all of them, whatever V.
__host__ __device__ inline size_t row_smem(int V) {
  const size_t rb = (size_t)NT * OWN * 4;
  (void)V;
  return rb > RWORK_BYTES ? rb : RWORK_BYTES;
}
static_assert((size_t)NT * OWN >= (size_t)F_MAXV + 3, "the staged row (with its alignment shift) fits");
static_assert(RWORK_BYTES >= 5 * 1024 + CAND_CAP * 8, "big-path scratch fits the work area");

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  return v;
}
__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(FULL, v, o);
    v = w > v ? w : v;
  }
  return v;
}
__device__ __forceinline__ unsigned long long warp_min_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(FULL, v, o);
    v = w < v ? w : v;
  }
  return v;
}
struct SumD { __device__ double operator()(double a, double b) const { return a + b; } };
struct MinF { __device__ float operator()(float a, float b) const { return fminf(a, b); } };

// Exclusive scan of one double per thread of the CTA; *total gets the sum.
__device__ __forceinline__ double block_exscan_f64(double v, double* red, double* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(FULL, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) red[warp] = x;
  csync();
  double wbase = 0.0, tot = 0.0;
#pragma unroll
  for (int w = 0; w < NWARP; ++w) {
    const double t = red[w];
    if (w < warp) wbase += t;
    tot += t;
  }
  csync();
  *total = tot;
  return wbase + x - v;
}

// Warp search over NB bins (PER = NB/32 per lane): first logical bin whose
// inclusive running sum exceeds `target`; *before_out = sum of the bins
// before it; *c_out = NB if none. Whole warp calls; one lane writes.
template <int PER, typename T, typename Get>
__device__ __forceinline__ void warp_find_bin_n(Get get, T target, int* c_out, T* before_out) {
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
  const unsigned bal = __ballot_sync(FULL, incl > target);
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
      if (run + loc[j] > target) { c = L * PER + j; before = run; break; }
      run += loc[j];
    }
    *c_out = c;
    *before_out = before;
  }
}

// Octave/sub-bin rank of an estimate p in (0, 1]: ((0x3F800000 - bits(p)) >>
// 15) = 256 b + s, where octave b holds p in (2^-(b+1), 2^-b] and the 256
// sub-bins s split it linearly in p; a larger rank is a smaller p. Clamped to
// the last (open) octave NOCT.
__device__ __forceinline__ int est_rank(float p) {
  const int r = (int)(0x3F800000u - __float_as_uint(p)) >> 15;
  return min(max(r, 0), NOCT * 256 + 255);
}
// |d| = |y - m_y| of an element whose estimate lies in octave b is below
// (b+1) ln 2 (up to the estimate's own tiny error); the open octave holds
// everything down to the clamp at -200.
__device__ __forceinline__ double oct_d(int b) { return b < NOCT ? 0.6932 * (b + 1) : 200.0; }

// Everything one sampled row's passes need.
struct RowCtx {
  int row, V, i0;            // i0: element index of this thread's first position
  float m_x, m_y, T, rT;     // rT = RN(1/T) (1 without temperature)
  bool do_t;
  double thr, u;
  unsigned long long xs, u53;
};
// fl(x / T), the reference's tempered value (sampling.cpp:16).
__device__ __forceinline__ float yex(const RowCtx& rc, float x) { return rc.do_t ? div_rn(x, rc.T, rc.rT) : x; }
// Estimate of y - m_y: one rounding of x * RN(1/T) - m_y, clamped at -200.
__device__ __forceinline__ float dest(const RowCtx& rc, float x) { return fmaxf(fmaf(x, rc.rT, -rc.m_y), -200.0f); }

// Unit roundoff of float.
constexpr double U24 = 5.9604644775390625e-08;

// Error bound of an estimated mass `mass` = sum of p~ over a set, where
// dmass >= sum of |d| p~ over the same set. Per element, with u = 2^-24 and
// |d| = |y - m_y|: the estimate d~ of y - m_y (one FMA from x, RN(1/T) and
// m_y) is within u(2|m_y| + 4|d|) of the reference's fl(fl(x/T) - m_y);
// __expf adds at most (2 + 1.2|d|) ulps (CUDA documents 2 + floor(|1.173 d|)),
// i.e. (4 + 2.4|d|)u relative; so |p~ - p| <= u(4 + 2|m_y| + 6.4|d|) p~. Float
// sums of at most nsum terms add nsum*u of their magnitude. Results that
// __expf flushes to zero (or the clamp at -200) hide at most 2^-125 each.
// 5% margin on the whole.
__device__ __forceinline__ double est_err(double mass, double dmass, float m_y, int nsum, int nelem) {
  return U24 * 1.05 * ((4.0 + 2.0 * fabs((double)m_y) + (double)nsum) * mass + 6.4 * dmass) +
         (double)nelem * 2.3509887016445750e-38;
}

// Hands a row to the general path (defer_kernel).
__device__ __forceinline__ void defer_row(const Args& a, int row) {
  const unsigned t = atomicAdd(&a.defer_cnt[0], 1u);
  a.defer_rows[t] = row;
  atomicAdd(&a.counters[C4S_CNT_DEFERRED], 1ull);
}

// ===========================================================================
// List kernel: one warp per row
// ===========================================================================

// Reduction scratch of a list job run by a whole CTA.
struct LRed {
  double d[NWARP];
  unsigned long long q[NWARP];
  int i[NWARP];
  int e;
  double x, y;
};

// A list job runs on one warp (short lists) or on the whole CTA (long ones);
// LG<CTA> gives its group size, rank, barrier and group-wide reductions. All
// members of the group call each function; every member gets the same result.
template <bool CTA>
struct LG {
  static constexpr int N = CTA ? NT : 32;
  __device__ static int rank() { return CTA ? (int)threadIdx.x : (int)(threadIdx.x & 31); }
  __device__ static void sync() {
    if (CTA) csync(); else __syncwarp();
  }
  __device__ static double sum(double v, LRed& R) {
    v = warp_sum_d(v);
    if (!CTA) return v;
    if ((threadIdx.x & 31) == 0) R.d[threadIdx.x >> 5] = v;
    csync();
    double s = 0.0;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) s += R.d[w];
    csync();
    return s;
  }
  __device__ static int add(int v, LRed& R) {
    v = __reduce_add_sync(FULL, v);
    if (!CTA) return v;
    if ((threadIdx.x & 31) == 0) R.i[threadIdx.x >> 5] = v;
    csync();
    int s = 0;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) s += R.i[w];
    csync();
    return s;
  }
  __device__ static unsigned long long qmin(unsigned long long v, LRed& R) {
    v = warp_min_u64(v);
    if (!CTA) return v;
    if ((threadIdx.x & 31) == 0) R.q[threadIdx.x >> 5] = v;
    csync();
    unsigned long long s = R.q[0];
#pragma unroll
    for (int w = 1; w < NWARP; ++w) s = R.q[w] < s ? R.q[w] : s;
    csync();
    return s;
  }
  __device__ static unsigned long long qmax(unsigned long long v, LRed& R) {
    v = warp_max_u64(v);
    if (!CTA) return v;
    if ((threadIdx.x & 31) == 0) R.q[threadIdx.x >> 5] = v;
    csync();
    unsigned long long s = R.q[0];
#pragma unroll
    for (int w = 1; w < NWARP; ++w) s = R.q[w] > s ? R.q[w] : s;
    csync();
    return s;
  }
  // Exclusive scan in rank order; *tot gets the group total.
  __device__ static int exscan_i(int v, LRed& R, int* tot) {
    const int lane = threadIdx.x & 31;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(FULL, x, o);
      if (lane >= o) x += y;
    }
    if (!CTA) {
      *tot = __shfl_sync(FULL, x, 31);
      return x - v;
    }
    const int warp = threadIdx.x >> 5;
    if (lane == 31) R.i[warp] = x;
    csync();
    int base = 0, t = 0;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) {
      if (w < warp) base += R.i[w];
      t += R.i[w];
    }
    csync();
    *tot = t;
    return base + x - v;
  }
  __device__ static double exscan_d(double v, LRed& R, double* tot) {
    const int lane = threadIdx.x & 31;
    double x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(FULL, x, o);
      if (lane >= o) x += y;
    }
    if (!CTA) {
      *tot = __shfl_sync(FULL, x, 31);
      return x - v;
    }
    const int warp = threadIdx.x >> 5;
    if (lane == 31) R.d[warp] = x;
    csync();
    double base = 0.0, t = 0.0;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) {
      if (w < warp) base += R.d[w];
      t += R.d[w];
    }
    csync();
    *tot = t;
    return base + x - v;
  }
  // Value of rank `src` (uniform) to every member.
  __device__ static int bcast_i(int v, int src, LRed& R) {
    if (!CTA) return __shfl_sync(FULL, v, src);
    if ((int)threadIdx.x == src) R.e = v;
    csync();
    const int r = R.e;
    csync();
    return r;
  }
  __device__ static void bcast_2d(double& a, double& b, int src, LRed& R) {
    if (!CTA) {
      a = __shfl_sync(FULL, a, src);
      b = __shfl_sync(FULL, b, src);
      return;
    }
    if ((int)threadIdx.x == src) { R.x = a; R.y = b; }
    csync();
    a = R.x;
    b = R.y;
    csync();
  }
};

// Ascending bitonic sort of np (power of two) keys by the group.
template <bool CTA>
__device__ void group_bitonic(unsigned long long* b, int np) {
  using G = LG<CTA>;
  for (int k = 2; k <= np; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = G::rank(); i < np; i += G::N) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long x = b[i], y = b[ixj];
          const bool up = (i & k) == 0;
          if ((x > y) == up) { b[i] = y; b[ixj] = x; }
        }
      }
      G::sync();
    }
  }
}

// Radix searches of a list job over the value keys that share `prefix` above
// bit b0 (8 bits per pass, histogram `hist` of 256 bins in shared memory).
// topk: the largest v with count(vkey >= v) >= k, i.e. the k-th largest key.
template <bool CTA>
__device__ __forceinline__ unsigned radix_kth(const unsigned* __restrict__ vk, int n, unsigned prefix, int b0, int k,
                                              unsigned long long* __restrict__ hist, LRed& R) {
  using G = LG<CTA>;
  unsigned* h = reinterpret_cast<unsigned*>(hist);
  const int lane = threadIdx.x & 31;
  int need = k;
  for (int hi = b0; hi >= 0;) {
    const int w = hi + 1 < 8 ? hi + 1 : 8;
    const int lo = hi - w + 1;
    const unsigned pmask = hi >= 31 ? 0u : ~((2u << hi) - 1u);
    for (int i = G::rank(); i < 256; i += G::N) h[i] = 0u;
    G::sync();
    for (int e = G::rank(); e < n; e += G::N) {
      const unsigned v = vk[e];
      if ((v & pmask) == prefix) atomicAdd(&h[(v >> lo) & 255u], 1u);
    }
    G::sync();
    if (!CTA || threadIdx.x < 32) {
      // lane l holds bins 8l..8l+7; suffix counts C(d) = #(digits >= d)
      unsigned c[8], s = 0u;
#pragma unroll
      for (int j = 0; j < 8; ++j) { c[j] = h[8 * lane + j]; s += c[j]; }
      unsigned above = s;                             // inclusive suffix over lanes >= lane
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned y = __shfl_down_sync(FULL, above, o);
        if (lane + o < 32) above += y;
      }
      unsigned run = above - s;                       // digits above this lane's bins
      int q = 0, dl = -1;
      unsigned nneed = 0u;
#pragma unroll
      for (int j = 7; j >= 0; --j) {
        run += c[j];                                  // C(8 lane + j)
        if (run >= (unsigned)need) {
          ++q;
          if (dl < 0) { dl = 8 * lane + j; nneed = (unsigned)need - (run - c[j]); }
        }
      }
      // the qualifying digits are 0..d*; d* is the largest, found on one lane
      const int D = __reduce_add_sync(FULL, q);
      const int ds = D > 0 ? D - 1 : 0;
      const unsigned src = __ballot_sync(FULL, dl == ds);
      const int sl = src ? __ffs(src) - 1 : 0;
      const unsigned nn = __shfl_sync(FULL, D > 0 ? nneed : (unsigned)need, sl);
      if (CTA) {
        if (threadIdx.x == 0) { R.e = ds; R.i[0] = (int)nn; }
      } else {
        prefix |= (unsigned)ds << lo;
        need = (int)nn;
      }
    }
    if (CTA) {
      csync();
      prefix |= (unsigned)R.e << lo;
      need = R.i[0];
      csync();
    }
    hi = lo - 1;
  }
  return prefix;
}

// mass: the largest v with base + sum(pv[e] : vkey(e) < v) <= Th (v = prefix if
// none), where base is the mass below the searched range. The bins add p in
// 2^-52 fixed point (native 64-bit shared atomics; p <= 1 and n <= 2048); the
// search only has to land on the crossing value, which the caller then checks
// with double sums and their error band.
template <bool CTA>
__device__ __forceinline__ unsigned radix_mass(const unsigned* __restrict__ vk, const double* __restrict__ pv, int n,
                                               unsigned prefix, int b0, double base, double Th,
                                               unsigned long long* __restrict__ hist, LRed& R) {
  using G = LG<CTA>;
  unsigned long long* h = hist;
  const int lane = threadIdx.x & 31;
  for (int hi = b0; hi >= 0;) {
    const int w = hi + 1 < 8 ? hi + 1 : 8;
    const int lo = hi - w + 1;
    const unsigned pmask = hi >= 31 ? 0u : ~((2u << hi) - 1u);
    for (int i = G::rank(); i < 256; i += G::N) h[i] = 0ull;
    G::sync();
    for (int e = G::rank(); e < n; e += G::N) {
      const unsigned v = vk[e];
      const double p = pv[e];
      if ((v & pmask) == prefix && p != 0.0)
        atomicAdd(&h[(v >> lo) & 255u], __double2ull_rn(p * 4503599627370496.0));
    }
    G::sync();
    if (!CTA || threadIdx.x < 32) {
      // lane l holds bins 8l..8l+7; E(d) = mass of digits < d
      double m[8], s = 0.0;
#pragma unroll
      for (int j = 0; j < 8; ++j) { m[j] = (double)h[8 * lane + j] * 2.220446049250313e-16; s += m[j]; }
      double incl = s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const double y = __shfl_up_sync(FULL, incl, o);
        if (lane >= o) incl += y;
      }
      double run = incl - s;
      int q = 0;
      double ed = 0.0;
      int dl = -1;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (base + run <= Th) { ++q; dl = 8 * lane + j; ed = run; }
        run += m[j];
      }
      const int D = __reduce_add_sync(FULL, q);
      const int ds = D > 0 ? D - 1 : 0;
      const unsigned src = __ballot_sync(FULL, dl == ds);
      const int sl = src ? __ffs(src) - 1 : 0;
      const double e = __shfl_sync(FULL, ed, sl);
      if (CTA) {
        if (threadIdx.x == 0) { R.e = ds; R.x = D > 0 ? e : 0.0; }
      } else {
        prefix |= (unsigned)ds << lo;
        base += D > 0 ? e : 0.0;
      }
    }
    if (CTA) {
      csync();
      prefix |= (unsigned)R.e << lo;
      base += R.x;
      csync();
    }
    hi = lo - 1;
  }
  return prefix;
}

// One list job. keys[0..n) (global): ckey(y, i) of the candidates in index
// order (list position = index order). The job stages their value keys into
// vk[] and computes their probabilities into pv[] (zero for candidates that
// top-k removes), both in shared memory, so that its passes stay on chip;
// pvg / sb (global) serve the rare exact fallback. Run by one warp (CTA =
// false) or by the whole CTA (long lists). With `refine` (the general kernel,
// after replacing an estimated tail by the exact one) a row that cannot be
// decided is not handed back: the caller finishes it on the general path.
// Returns whether the row is finished.
template <bool CTA>
__device__ __forceinline__ bool list_job(const Args& a, int row, RowJob& J,
                                         const unsigned long long* __restrict__ keys, unsigned long long* sb,
                                         unsigned* __restrict__ vk, double* __restrict__ pv,
                                         unsigned long long* __restrict__ hist, bool refine, LRed& R) {
  using G = LG<CTA>;
  const int r0 = G::rank();
  constexpr int GN = G::N;
  const int n = J.n, V = a.V, k = J.k;
  const float m_y = J.m_y;
  const bool k0 = J.kind == JOB_K0;
  const bool forced = (a.debug & C4S_DEBUG_FORCE_BINS) != 0;
  auto hand_back = [&](int st) {
    if (r0 == 0 && !refine) {
      J.status = st;
      defer_row(a, row);
    }
  };
  // stage the value keys: eight loads in flight per member
  unsigned long long vmin = ~0ull, vmax = 0ull;
  for (int e0 = r0; e0 < n; e0 += 8 * GN) {
    unsigned v[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int e = e0 + q * GN;
      v[q] = e < n ? (unsigned)(__ldcg(keys + e) >> 32) : 0u;
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int e = e0 + q * GN;
      if (e < n) {
        vk[e] = v[q];
        vmin = v[q] < vmin ? v[q] : vmin;
        vmax = v[q] > vmax ? v[q] : vmax;
      }
    }
  }
  vmin = G::qmin(vmin, R);
  vmax = G::qmax(vmax, R);
  G::sync();
  // no-top-k list: everything below it must be strictly smaller in value
  if (k0 && J.ykex >= vmin) { hand_back(RES_DEFER); return false; }
  if (k0 && !refine && (a.debug & C4S_DEBUG_FORCE_REFINE)) { hand_back(RES_REFINE); return false; }

  // ---- top-k threshold: the k-th largest value key (sampling.cpp:30-40) ----
  unsigned tk = (unsigned)vmin;
  if (k > 0 && k < n && vmin != vmax) {
    const int b0 = 31 - __clz((unsigned)(vmin ^ vmax));
    const unsigned v = b0 >= 31 ? 0u : ((unsigned)vmax & ~((2u << b0) - 1u));
    tk = radix_kth<CTA>(vk, n, v, b0, k, hist, R);
  }

  // ---- exact probabilities of the survivors (sampling.cpp:52-55) ----
  double ps = 0.0;
  int ns = 0;
  unsigned long long smin = ~0ull, elast = 0ull;
#pragma unroll 4
  for (int e = r0; e < n; e += GN) {
    const unsigned v = vk[e];
    double p = 0.0;
    if (v >= tk) {
      p = exp((double)__fsub_rn(fkey_inv(v), m_y));    // prob(): the reference's exp((double)(y - max))
      ++ns;
      smin = v < smin ? v : smin;
    }
    if (v == (unsigned)vmax) elast = e;               // last (largest-index) maximum
    pv[e] = p;
    ps += p;
  }
  ps = G::sum(ps, R);
  ns = G::add(ns, R);
  smin = G::qmin(smin, R);
  const unsigned long long kmax = keys[G::qmax(elast, R)];   // the largest survivor key
  G::sync();

  // ---- top-p (sampling.cpp:42-71) ----
  const double thr = J.thr;
  const double tail = J.tail;
  const double St = tail + ps;
  unsigned long long kst = 0ull;
  bool exact_tp = false;
  if (thr < 0.0) {
    kst = 0ull;                                       // p > 1: nothing removed
  } else if (thr == 0.0) {
    unsigned long long mk0 = KEY_MAX;                 // p == 1: only zero probabilities go
    for (int e = r0; e < n; e += GN)
      if (vk[e] >= tk && pv[e] > 0.0) mk0 = keys[e] < mk0 ? keys[e] : mk0;
    kst = G::qmin(mk0, R);
  } else {
    const double Th = thr * St;
    // G(c) = tail + sum of p over value keys < c (removed candidates have p = 0);
    // the largest c with G(c) <= Th is the value of the crossing element
    const unsigned smin32 = (unsigned)smin, vmax32 = (unsigned)vmax;
    const int b0 = (smin32 == vmax32) ? -1 : 31 - __clz(smin32 ^ vmax32);
    unsigned v = b0 < 0 ? smin32 : (b0 >= 31 ? 0u : (vmax32 & ~((2u << b0) - 1u)));
    v = radix_mass<CTA>(vk, pv, n, v, b0, tail, Th, hist, R);
    double Gs = 0.0, Mg = 0.0;
    int cg = 0;
    for (int e = r0; e < n; e += GN) {
      const unsigned ve = vk[e];
      if (ve < v) Gs += pv[e];
      else if (ve == v && ve >= tk) { Mg += pv[e]; ++cg; }
    }
    Gs = tail + G::sum(Gs, R);
    Mg = G::sum(Mg, R);
    cg = G::add(cg, R);
    if (cg > 0 && Gs <= Th && Gs + Mg > Th) {
      // crossing inside the value group v; equal values have equal p and
      // keep index order: the t-th member of the group in index order
      const double pg = Mg / cg;
      int t = 1;
      if (cg > 1) {
        const double q = floor((Th - Gs) / pg) + 1.0;
        t = (int)fmin(fmax(q, 1.0), (double)cg);
      }
      int es = 0, acc = 0;
      for (int e0 = 0; e0 < n; e0 += GN) {
        const int e = e0 + r0;
        const bool m = e < n && vk[e] == v;
        int tot;
        const int before = G::exscan_i(m ? 1 : 0, R, &tot);
        if (t <= acc + tot) {
          const bool me = m && acc + before + 1 == t;
          es = (int)G::qmin(me ? (unsigned long long)e : ~0ull, R);
          break;
        }
        acc += tot;
      }
      const double before = Gs + (double)(t - 1) * pg, cur = Gs + (double)t * pg;
      const double bd = 2.0 * ((4.0 * (k0 ? V : ns) + 16.0) * U53 * St) + 2.0 * J.tail_err;
      kst = keys[es];
      exact_tp = !(before <= Th - bd && cur > Th + bd);
    } else {
      kst = KEY_MAX;                                  // no crossing: only the kept maximum
      exact_tp = true;
    }
    exact_tp = exact_tp || forced;
  }
  if (exact_tp) {
    if (k0) {                                         // the tail is exact only after a refine
      if (!refine) hand_back(RES_REFINE);
      return false;
    }
    // the reference's sequential sums over the survivors in ascending order
    int base = 0;
    for (int e0 = 0; e0 < n; e0 += GN) {
      const int e = e0 + r0;
      const bool sv = e < n && vk[e] >= tk;
      int tot;
      const int pos = G::exscan_i(sv ? 1 : 0, R, &tot);
      if (sv) sb[base + pos] = keys[e];
      base += tot;
    }
    int np = 1;
    while (np < ns) np <<= 1;
    for (int s = ns + r0; s < np; s += GN) sb[s] = KEY_MAX;
    G::sync();
    group_bitonic<CTA>(sb, np);
    for (int s = r0; s < ns; s += GN) pv[s] = prob(fkey_inv((unsigned)(sb[s] >> 32)), m_y);
    G::sync();
    int js = ns;
    if (r0 == 0) {
      double sum = 0.0;
      for (int s = 0; s < ns; ++s) sum = __dadd_rn(sum, pv[s]);
      double cum = 0.0;
      for (int s = 0; s < ns; ++s) {
        cum = __dadd_rn(cum, __ddiv_rn(pv[s], sum));
        if (!(cum <= thr)) { js = s; break; }
      }
      atomicAdd(&a.counters[C4S_CNT_TOPP_EXACT_FALLBACK], 1ull);
    }
    js = G::bcast_i(js, 0, R);
    kst = js < ns ? sb[js] : KEY_MAX;
    G::sync();
    // probabilities by position again, for the draw
    for (int e = r0; e < n; e += GN) pv[e] = vk[e] >= tk ? prob(fkey_inv(vk[e]), m_y) : 0.0;
    G::sync();
  }
  kst = kst < kmax ? kst : kmax;                      // min_tokens_to_keep = 1

  // ---- the draw (text2semantic.cpp:150-165); index order = position order ----
  // keys[e] >= kst, read from global memory only for the value tied with kst
  const unsigned kv = (unsigned)(kst >> 32);
  auto kept = [&](int e) {
    if (e >= n) return false;
    const unsigned v = vk[e];
    return v >= tk && (v > kv || (v == kv && keys[e] >= kst));
  };
  int tok = 0;
  if (J.u53 != 0ull) {
    const double u = J.u;
    double s2 = 0.0;
    int nk = 0;
    for (int e = r0; e < n; e += GN)
      if (kept(e)) { s2 += pv[e]; ++nk; }
    s2 = G::sum(s2, R);
    nk = G::add(nk, R);
    const double r = u * s2;
    double carry = 0.0, prev = 0.0, cur = 0.0;
    int found = -1;
    for (int e0 = 0; e0 < n; e0 += GN) {
      const int e = e0 + r0;
      const bool kp = kept(e);
      const double x = kp ? pv[e] : 0.0;
      double tot;
      const double incl = carry + G::exscan_d(x, R, &tot) + x;
      const unsigned long long hit = G::qmin(kp && incl >= r ? (unsigned long long)e : ~0ull, R);
      if (hit != ~0ull) {
        found = (int)hit;
        prev = incl - x;
        cur = incl;
        G::bcast_2d(prev, cur, found - e0, R);
        break;
      }
      carry += tot;
    }
    const double bd2 = 2.0 * ((4.0 * nk + 16.0) * U53 * s2);
    if (!forced && found >= 0 && prev < r - bd2 && cur > r + bd2) {
      tok = ckey_idx(keys[found]);
    } else {
      // the reference's sequential sums in index order
      int t = V - 1;
      if (r0 == 0) {
        double sum = 0.0;
        for (int e = 0; e < n; ++e)
          if (kept(e)) sum = __dadd_rn(sum, pv[e]);
        const double rr = __dmul_rn(u, sum);
        double acc = 0.0;
        for (int e = 0; e < n; ++e) {
          if (kept(e)) {
            acc = __dadd_rn(acc, pv[e]);
            if (rr <= acc) { t = ckey_idx(keys[e]); break; }
          }
        }
        atomicAdd(&a.counters[C4S_CNT_DRAW_EXACT_FALLBACK], 1ull);
      }
      tok = G::bcast_i(t, 0, R);
    }
  }
  if (r0 == 0) {
    a.out_ids[row] = tok;
    a.rng[row] = J.xs;
    J.kstar = kst;
    J.thresh_key = k > 0 ? tk : 0u;
    J.status = RES_DONE;
  }
  G::sync();
  return true;
}

// List kernel dynamic shared memory: per warp a list of up to LW_CAP entries
// (staged value keys, probabilities) and a radix histogram; once the warps are
// done, the same area holds one long list (up to LCAP) worked by the whole CTA.
constexpr int LW_CAP = 1024;                  // longest list one warp takes
constexpr size_t LW_VK = 0, LW_PV = (size_t)LW_CAP * 4, LW_HIST = LW_PV + (size_t)LW_CAP * 8;
constexpr size_t LW_BYTES = LW_HIST + 256 * 8;            // per warp
constexpr size_t LB_VK = 0, LB_PV = (size_t)LCAP * 4, LB_HIST = LB_PV + (size_t)LCAP * 8;
constexpr size_t LIST_SMEM = (size_t)LIST_WARPS * LW_BYTES;
static_assert(LB_HIST + 256 * 8 <= LIST_SMEM, "a long list fits the warps' areas");

// Short lists: one warp each. Long lists (the row kernel queued them): CTAs
// take them one at a time from a shared counter once their warps are done.
__global__ void __launch_bounds__(32 * LIST_WARPS, 2) list_kernel(Args a) {
  static_assert(32 * LIST_WARPS == NT, "the list kernel's CTA barrier counts NT threads");
  extern __shared__ __align__(16) unsigned char lsm[];
  __shared__ LRed R;
  __shared__ int next;
  const int w = threadIdx.x >> 5;
  const int row = blockIdx.x * LIST_WARPS + w;
  if (row < a.B) {
    RowJob& J = a.jobs[row];
    const int kind = J.kind;
    if ((kind == JOB_TOPK || kind == JOB_K0) && J.n <= LW_CAP) {
      unsigned char* wa = lsm + (size_t)w * LW_BYTES;
      const size_t o = (size_t)row * LCAP;
      list_job<false>(a, row, J, a.lkeys + o, a.lsb + o, reinterpret_cast<unsigned*>(wa + LW_VK),
                      reinterpret_cast<double*>(wa + LW_PV), reinterpret_cast<unsigned long long*>(wa + LW_HIST),
                      false, R);
    }
  }
  const unsigned nbig = *reinterpret_cast<volatile unsigned*>(&a.defer_cnt[3]);
  for (;;) {
    csync();                                        // the warps' lists are done with the area
    if (threadIdx.x == 0) next = (int)atomicAdd(&a.defer_cnt[4], 1u);
    csync();
    const int t = next;
    if (t >= (int)nbig) break;
    const int r = a.big_rows[t];
    const size_t o = (size_t)r * LCAP;
    list_job<true>(a, r, a.jobs[r], a.lkeys + o, a.lsb + o, reinterpret_cast<unsigned*>(lsm + LB_VK),
                   reinterpret_cast<double*>(lsm + LB_PV), reinterpret_cast<unsigned long long*>(lsm + LB_HIST),
                   false, R);
  }
}

// ===========================================================================
// Row kernel
// ===========================================================================

// This thread's block of the staged row into registers: buffer positions
// [36t, 36t+36) (element index = position - shift); positions outside the row
// read as -inf (never a candidate, mass 0).
__device__ __forceinline__ void load_block(const float* rowbuf, int shift, int V, float (&x)[OWN]) {
  const int p0 = threadIdx.x * OWN;
  const int i0 = p0 - shift;
  const float4* r4 = reinterpret_cast<const float4*>(rowbuf + p0);
  if (i0 >= 0 && i0 + OWN <= V) {                  // every position holds an element
#pragma unroll
    for (int q = 0; q < OWN / 4; ++q) {
      const float4 v = r4[q];
      x[4 * q] = v.x;
      x[4 * q + 1] = v.y;
      x[4 * q + 2] = v.z;
      x[4 * q + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int q = 0; q < OWN / 4; ++q) {
      const float4 v = r4[q];
      const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int r = 0; r < 4; ++r) x[4 * q + r] = (unsigned)(i0 + 4 * q + r) < (unsigned)V ? vv[r] : -INFINITY;
    }
  }
}

// x[j] for a run-time j (a select chain: registers cannot be indexed).
__device__ __forceinline__ float pick(const float (&x)[OWN], int j) {
  float v = x[0];
#pragma unroll
  for (int jj = 1; jj < OWN; ++jj) v = (j == jj) ? x[jj] : v;
  return v;
}

// Writes a row of processed logits from a copy of this thread's elements: y,
// or -inf where the top-k threshold key or K* removes it. Out of line: it only
// runs when processed logits are requested.
__device__ __noinline__ void write_row(const Args& a, const RowCtx& rc, const float* x, bool temper,
                                       unsigned thresh_key, unsigned long long kst) {
  float* o = a.out_logits + (long long)rc.row * a.out_ld;
  for (int j = 0; j < OWN; ++j) {
    const int i = rc.i0 + j;
    if ((unsigned)i < (unsigned)rc.V) {
      const float y = temper ? yex(rc, x[j]) : x[j];
      const bool masked = fkey(y) < thresh_key || (y > -INFINITY && ckey(y, i) < kst);
      o[i] = masked ? -INFINITY : y;
    }
  }
}
// As write_row, from the registers (through a local copy, so that x itself
// stays in registers).
__device__ __forceinline__ void write_row_regs(const Args& a, const RowCtx& rc, const float (&x)[OWN], bool temper) {
  float xc[OWN];
#pragma unroll
  for (int j = 0; j < OWN; ++j) xc[j] = x[j];
  write_row(a, rc, xc, temper, 0u, 0ull);
}

// Candidate of the big path: a row element of the crossing octave.
struct Cand {
  float x;
  int pos;                   // owner thread * OWN + j
};

// The kw-th largest (1 <= kw <= 64) of the warp's 64 keys (a and b of each
// lane): bitonic sort of two keys per lane (blocked layout).
__device__ __forceinline__ unsigned warp_kth_largest64(unsigned a, unsigned b, int kw) {
  const int lane = threadIdx.x & 31;
  unsigned v0 = a, v1 = b;
#pragma unroll
  for (int k2 = 2; k2 <= 64; k2 <<= 1) {
#pragma unroll
    for (int jj = k2 >> 1; jj > 0; jj >>= 1) {
      if (jj == 1) {
        const bool up = ((2 * lane) & k2) == 0;
        const unsigned lo = min(v0, v1), hi = max(v0, v1);
        v0 = up ? lo : hi;
        v1 = up ? hi : lo;
      } else {
        const int lj = jj >> 1;
        const unsigned o0 = __shfl_xor_sync(FULL, v0, lj), o1 = __shfl_xor_sync(FULL, v1, lj);
        const int q0 = 2 * lane, q1 = 2 * lane + 1;
        const bool m0 = ((q0 & jj) == 0) == ((q0 & k2) == 0);
        const bool m1 = ((q1 & jj) == 0) == ((q1 & k2) == 0);
        v0 = m0 ? min(v0, o0) : max(v0, o0);
        v1 = m1 ? min(v1, o1) : max(v1, o1);
      }
    }
  }
  const int pos = 64 - kw;                         // ascending order
  const unsigned w0 = __shfl_sync(FULL, v0, pos >> 1), w1 = __shfl_sync(FULL, v1, pos >> 1);
  return (pos & 1) ? w1 : w0;
}
// The kw-th largest (1 <= kw <= 32) of the warp's 32 keys.
__device__ __forceinline__ unsigned warp_kth_largest32(unsigned key, int kw) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k2 = 2; k2 <= 32; k2 <<= 1) {
#pragma unroll
    for (int jj = k2 >> 1; jj > 0; jj >>= 1) {
      const unsigned o = __shfl_xor_sync(FULL, key, jj);
      const bool keep_min = (((lane & jj) == 0) == ((lane & k2) == 0));
      key = keep_min ? (o < key ? o : key) : (o > key ? o : key);
    }
  }
  return __shfl_sync(FULL, key, 32 - kw);
}

// Header fields common to both list job kinds (thread 0).
__device__ __forceinline__ void fill_job(RowJob& J, const RowCtx& rc, int kind, int n, int k) {
  J.kind = kind;
  J.n = n;
  J.k = k;
  J.status = RES_DONE;
  J.m_y = rc.m_y;
  J.thresh_key = 0u;
  J.thr = rc.thr;
  J.u = rc.u;
  J.u53 = rc.u53;
  J.xs = rc.xs;
  J.kstar = 0ull;
}

// A list longer than one list-kernel warp takes goes to the CTA-wide queue.
__device__ __forceinline__ void queue_long_list(const Args& a, int row, int n) {
  if (n > LW_CAP) a.big_rows[atomicAdd(&a.defer_cnt[3], 1u)] = row;
}

// Writes the keys of this thread's candidates (bit j of mask: position j)
// into the row's list from wpos on, in index order.
__device__ __forceinline__ void write_keys(unsigned long long* keys, const RowCtx& rc, const float (&x)[OWN],
                                           unsigned long long mask, int wpos) {
  while (mask) {
    const int j = __ffsll((long long)mask) - 1;
    mask &= mask - 1ull;
    keys[wpos++] = ckey(yex(rc, pick(x, j)), rc.i0 + j);
  }
}

// As write_keys, from a local copy of the elements (indexable).
__device__ __forceinline__ void write_keys_mem(unsigned long long* keys, const RowCtx& rc, const float* x,
                                           unsigned long long mask, int wpos) {
  while (mask) {
    const int j = __ffsll((long long)mask) - 1;
    mask &= mask - 1ull;
    keys[wpos++] = ckey(yex(rc, x[j]), rc.i0 + j);
  }
}

enum { ROW_DONE = 0, ROW_GENERAL = 1 };

// Octave totals of a row without top-k and its crossing octave.
struct K0Oct {
  double Se, Ee, Th, rnd, cum, Eb;
  int bc;                          // crossing octave; -1: top_p > 1, everything is kept
};

// The big path of a row without top-k, after its octave histogram (columns
// still in the work area): sub-bins and candidates of the crossing octave, an
// exact sort of the crossing sub-bin, then the draw over per-thread survivor
// masses. Out of line: only rows whose crossing list would be too long.
__device__ __noinline__ int k0_big(const Args& a, const RowCtx& rc, const float* x, unsigned char* work, Shared& S,
                                   bool forced, const K0Oct& O) {
  const int V = rc.V, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = rc.row;
  const float m_y = rc.m_y;
  const double thr = rc.thr;
  const int bc = O.bc;
  const double Se = O.Se, Ee = O.Ee, Th = O.Th, rnd = O.rnd, cum = O.cum, Eb = O.Eb;
  // survivor mass of this thread's elements in the octaves above the crossing one
  float hi = 0.0f;
  for (int j = 0; j < OWN; ++j) {
    const float p = __expf(dest(rc, x[j]));
    if (bc < 0 || (est_rank(p) >> 8) < bc) hi += p;
  }
  unsigned long long kst = 0ull;
  int fc = -1;                                    // crossing rank: octave * 256 + sub-bin
  double Ed = Ee;                                 // |d| mass bound of the survivors
  if (bc >= 0) {
    float* SBm = reinterpret_cast<float*>(work);
    unsigned* SBc = reinterpret_cast<unsigned*>(work + 1024);
    unsigned long long* ws = reinterpret_cast<unsigned long long*>(work + 2048);
    double* wpv = reinterpret_cast<double*>(work + 2048 + BIG_SORT * 8);
    float* acc2 = reinterpret_cast<float*>(work + 2048 + BIG_SORT * 16);
    Cand* cand = reinterpret_cast<Cand*>(work + 5 * 1024);
    SBm[tid] = 0.0f;
    SBc[tid] = 0u;
    acc2[tid] = 0.0f;
    if (tid == 0) { S.slot = 0; S.slot2 = 0; }
    csync();
    // sub-bins of the crossing octave and its elements
    float xdeep = -INFINITY, xhigh = INFINITY;
#pragma unroll
    for (int j = 0; j < OWN; ++j) {
      const float p = __expf(dest(rc, x[j]));
      const int rk = est_rank(p);
      const int ob = rk >> 8;
      if (ob == bc) {
        atomicAdd(&SBm[rk & 255], p);
        atomicAdd(&SBc[rk & 255], 1u);
        const int sl = atomicAdd(&S.slot, 1);
        if (sl < CAND_CAP) cand[sl] = Cand{x[j], tid * OWN + j};
      } else if (ob > bc) {
        xdeep = fmaxf(xdeep, x[j]);
      } else {
        xhigh = fminf(xhigh, x[j]);
      }
    }
    csync();
    if (warp == 0)
      warp_find_bin_n<8, float>([&](int jb) { return SBm[255 - jb]; }, (float)(Th - cum), &S.c, &S.fbefore);
    csync();
    const int ncand = S.slot;
    if (S.c >= 256 || ncand > CAND_CAP) return ROW_GENERAL;
    const int c2 = 255 - S.c;
    const int nc = (int)SBc[c2];
    if (nc > BIG_SORT || nc == 0) return ROW_GENERAL;
    fc = bc * 256 + c2;
    const double before = cum + (double)S.fbefore;
    // the crossing sub-bin with exact keys; the nearest values outside it
    float xb = xdeep, xa = xhigh;
    const int ishift = rc.i0 - tid * OWN;         // element index = position + ishift
    for (int e = tid; e < ncand; e += NT) {
      const Cand cd = cand[e];
      const int sub = est_rank(__expf(dest(rc, cd.x))) & 255;
      if (sub == c2) {
        const int sl = atomicAdd(&S.slot2, 1);
        if (sl < BIG_SORT) ws[sl] = ckey(yex(rc, cd.x), cd.pos + ishift);
      } else if (sub > c2) {
        xb = fmaxf(xb, cd.x);
      } else {
        xa = fminf(xa, cd.x);
      }
    }
    xb = block_reduce(xb, MaxF(), S.redf);
    xa = block_reduce(xa, MinF(), S.redf);
    if (warp == 0) {
      warp_sort(ws, nc);
      const unsigned klo = (unsigned)(ws[0] >> 32), khi = (unsigned)(ws[nc - 1] >> 32);
      // values outside the sub-bin must order strictly outside it
      const bool ok = (xb == -INFINITY || fkey(yex(rc, xb)) < klo) && (xa == INFINITY || fkey(yex(rc, xa)) > khi);
      for (int e = lane; e < nc; e += 32) wpv[e] = prob(fkey_inv((unsigned)(ws[e] >> 32)), m_y);
      __syncwarp();
      if (lane == 0) {
        // error bounds: the estimated mass below the crossing and the estimated total
        const double eb = est_err(before, Eb + (double)S.fbefore * oct_d(bc), m_y, 36 + ncand, V);
        const double bd = eb + thr * est_err(Se, Ee, m_y, 36 + ncand, V) + rnd;
        int e = -1;
        double prev = 0.0, curv = 0.0, run = before;
        for (int t = 0; t < nc; ++t) {
          if (run + wpv[t] > Th) { e = t; prev = run; curv = run + wpv[t]; break; }
          run += wpv[t];
        }
        S.defer = ok ? 0 : 1;
        S.done = (ok && e >= 0 && prev <= Th - bd && curv > Th + bd && !forced) ? 1 : 0;
        S.kp = e >= 0 ? ws[e] : KEY_MAX;
      }
    }
    csync();
    if (S.defer) return ROW_GENERAL;
    if (!S.done) {
      // exact sums over the row decide among the sub-bin's elements
      double se = 0.0, be = 0.0;
#pragma unroll
      for (int j = 0; j < OWN; ++j) {
        const double p = prob(yex(rc, x[j]), m_y);   // 0 for -inf
        se += p;
        if (est_rank(__expf(dest(rc, x[j]))) > fc) be += p;
      }
      se = block_reduce(se, SumD(), S.redd);
      be = block_reduce(be, SumD(), S.redd);
      if (tid == 0) {
        const double Te = thr * se, bde = 2.0 * ((4.0 * V + 16.0) * U53 * se);
        int e = -1;
        double prev = 0.0, curv = 0.0, run = be;
        for (int t = 0; t < nc; ++t) {
          if (run + wpv[t] > Te) { e = t; prev = run; curv = run + wpv[t]; break; }
          run += wpv[t];
        }
        S.defer = (e >= 0 && prev <= Te - bde && curv > Te + bde) ? 0 : 1;
        S.kp = e >= 0 ? ws[e] : KEY_MAX;
        atomicAdd(&a.counters[C4S_CNT_TOPP_EXACT_FALLBACK], 1ull);
      }
      csync();
      if (S.defer) return ROW_GENERAL;
    }
    kst = S.kp;
    // survivors inside the crossing octave, added to their owners' masses
    for (int e = tid; e < ncand; e += NT) {
      const Cand cd = cand[e];
      const float p = __expf(dest(rc, cd.x));
      const int sub = est_rank(p) & 255;
      if (sub < c2 || (sub == c2 && ckey(yex(rc, cd.x), cd.pos + ishift) >= kst)) atomicAdd(&acc2[cd.pos / OWN], p);
    }
    csync();
    hi += acc2[tid];
    Ed = 0.0;
    for (int b = 0; b <= bc; ++b) Ed += S.oct[b] * oct_d(b);
    if (tid == 0) atomicAdd(&a.counters[C4S_CNT_TOPP_BINNED], 1ull);
  }

  // ---- the draw: index-order prefix over per-thread survivor masses ----
  auto survives = [&](float xv, int i, float p) {
    if (fc < 0) return true;
    const int rk = est_rank(p);
    return rk < fc || (rk == fc && ckey(yex(rc, xv), i) >= kst);
  };
  int tok = 0;
  if (rc.u53 != 0ull) {
    bool done = false;
    for (int pass = forced ? 1 : 0; pass < 2 && !done; ++pass) {
      const bool exact = pass == 1;
      double loc = (double)hi;
      if (exact) {
        loc = 0.0;
#pragma unroll
        for (int j = 0; j < OWN; ++j)
          if (survives(x[j], rc.i0 + j, __expf(dest(rc, x[j])))) loc += prob(yex(rc, x[j]), m_y);
      }
      if (tid == 0) S.tok = -1;
      double Sk;
      const double base = block_exscan_f64(loc, S.redd, &Sk);
      // per-thread masses: <= 36-term column sums, <= 25 of them, <= 36 atomics
      const double Ek = exact ? 0.0 : est_err(Sk, Ed, m_y, 97, V);
      const double rq = rc.u * Sk;
      const double bd = 2.0 * Ek + 2.0 * ((4.0 * V + 16.0) * U53 * Sk);
      if (base < rq && base + loc >= rq) {
        // the crossing thread sums its own survivors in index order
        double run = 0.0;
        float runf = 0.0f;
        int found = -1;
        double fprev = 0.0, fcur = 0.0;
#pragma unroll
        for (int j = 0; j < OWN; ++j) {
          if (found < 0) {
            const float p = __expf(dest(rc, x[j]));
            if (x[j] > -INFINITY && survives(x[j], rc.i0 + j, p)) {
              double bef, aft;
              if (exact) { bef = run; run += prob(yex(rc, x[j]), m_y); aft = run; }
              else { bef = (double)runf; runf += p; aft = (double)runf; }
              if (base + aft >= rq) { found = rc.i0 + j; fprev = base + bef; fcur = base + aft; }
            }
          }
        }
        if (found >= 0) { S.tok = found; S.d1 = fprev; S.d2 = fcur; }
      }
      csync();
      const bool ok = Sk > 0.0 && S.tok >= 0 && S.d1 < rq - bd && S.d2 > rq + bd;
      const int t = S.tok;
      csync();
      if (ok) { tok = t; done = true; }
      else if (!exact && tid == 0) atomicAdd(&a.counters[C4S_CNT_DRAW_EXACT_FALLBACK], 1ull);
    }
    if (!done) return ROW_GENERAL;
  }
  if (tid == 0) {
    a.out_ids[row] = tok;
    a.rng[row] = rc.xs;
    a.jobs[row].kind = JOB_NONE;
    atomicAdd(&a.counters[C4S_CNT_DRAW_ROWPASS], 1ull);
  }
  if (a.out_logits) write_row(a, rc, x, true, 0u, kst);
  csync();
  return ROW_DONE;
}

// Fixed-point octave mass of an estimate p (its octave b = est_rank(p) >> 8):
// p * 2^(b+20), truncated, from the float's bits. Truncation loses less than
// 2^-(b+20) per element, i.e. below 2^-19 of any element in octaves < NOCT.
__device__ __forceinline__ unsigned oct_fix(float p, int b) {
  const unsigned u = __float_as_uint(p);
  const int sh = 130 - (int)(u >> 23) - b;        // 23 - 20 - (exponent + b)
  const unsigned m = (u & 0x007fffffu) | 0x00800000u;
  return (u == 0u || sh > 31) ? 0u : (m >> max(sh, 0));
}

// One sampled or greedy row whose penalised elements are in x (this thread's
// positions; `shift` is the row's misalignment in elements).
__device__ __forceinline__ int row_body(const Args& a, int row, const MetaSlot& M, const float (&x)[OWN], int shift,
                                        unsigned char* work, Shared& S) {
  const int V = a.V;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int i0 = tid * OWN - shift;
  const c4s_row_params P = M.P;
  const int k = P.top_k;
  const bool do_k = k > 0 && k < V;
  // top-k above 64: the two largest of each thread seed the list
  const bool two = !P.greedy && do_k && k > 64;

  // ---- row max and per-thread maxima ----
  float tm = -INFINITY, t2 = -INFINITY;
  if (two) {
#pragma unroll
    for (int j = 0; j < OWN; ++j) {
      t2 = fmaxf(t2, fminf(tm, x[j]));
      tm = fmaxf(tm, x[j]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < OWN; ++j) tm = fmaxf(tm, x[j]);
  }
  {
    const unsigned km = __reduce_max_sync(FULL, fkey(tm));
    if (lane == 0) S.redu[warp] = km;
  }
  csync();
  unsigned kall = S.redu[0];
#pragma unroll
  for (int w = 1; w < NWARP; ++w) kall = kall > S.redu[w] ? kall : S.redu[w];
  const float m_x = fkey_inv(kall);
  csync();

  RowCtx rc;
  rc.row = row; rc.V = V; rc.i0 = i0;
  rc.T = P.temperature;
  rc.do_t = !(rc.T == 1.0f || rc.T <= 0.0f);

  // ---- greedy: first index of the max (sampling.cpp:73-76) ----
  if (P.greedy) {
    unsigned cand = 0xffffffffu;
    if (m_x > -INFINITY && tm == m_x) {
#pragma unroll
      for (int j = 0; j < OWN; ++j)
        if (x[j] == m_x && (unsigned)(i0 + j) < cand) cand = (unsigned)(i0 + j);
    }
    cand = __reduce_min_sync(FULL, cand);
    if (lane == 0) S.redu[warp] = cand;
    csync();
    if (tid == 0) {
      unsigned b = S.redu[0];
      for (int w = 1; w < NWARP; ++w) b = S.redu[w] < b ? S.redu[w] : b;
      a.out_ids[row] = b == 0xffffffffu ? 0 : (int)b;
      a.jobs[row].kind = JOB_NONE;
    }
    if (a.out_logits) write_row_regs(a, rc, x, false);
    csync();
    return ROW_DONE;
  }

  // ---- sampled rows: preconditions ----
  if (!(m_x > -INFINITY && m_x < INFINITY)) return ROW_GENERAL;
  rc.m_x = m_x;
  rc.m_y = rc.do_t ? __fdiv_rn(m_x, rc.T) : m_x;
  rc.rT = rc.do_t ? __frcp_rn(rc.T) : 1.0f;
  if (!(fabsf(rc.m_y) < 262144.0f)) return ROW_GENERAL;
  if (P.min_tokens_to_keep != 1) return ROW_GENERAL;
  if (a.debug & C4S_DEBUG_FORCE_EXACT) return ROW_GENERAL;
  const bool forced = (a.debug & C4S_DEBUG_FORCE_BINS) != 0;
  rc.thr = __dsub_rn(1.0, (double)P.top_p);
  {
    unsigned long long xs = M.rng;
    xs ^= xs << 13; xs ^= xs >> 7; xs ^= xs << 17;
    rc.xs = xs;
    rc.u53 = xs >> 11;
    rc.u = (double)rc.u53 * 1.1102230246251565e-16;   // (x>>11) / 2^53, exact
  }
  if (!do_k) {
    // ---- rows without top-k (top-p over the whole row, sampling.cpp:42-71) ----
    if (rc.thr == 0.0) return ROW_GENERAL;
    // octave histogram of the estimates: per-warp fixed-point bins (exact adds)
    unsigned* Hw = reinterpret_cast<unsigned*>(work);
    Hw[warp * 32 + lane] = 0u;
    __syncwarp();
#pragma unroll
    for (int j = 0; j < OWN; ++j) {
      const float p = __expf(dest(rc, x[j]));
      const int b = est_rank(p) >> 8;
      atomicAdd(&Hw[warp * 32 + b], oct_fix(p, b));
    }
    csync();
    // every warp: lane b holds octave b's mass; suffix sums give the mass below
    // each octave, ballots the crossing octave and the list's last octave
    double o = 0.0;
    if (lane <= NOCT) {
      unsigned long long qs = 0ull;
#pragma unroll
      for (int w = 0; w < NWARP; ++w) qs += Hw[w * 32 + lane];
      o = ldexp((double)qs, -(lane + 20));
    }
    const double w = o * oct_d(lane <= NOCT ? lane : NOCT);
    double suf = o, wsuf = w;                       // sums over octaves >= lane
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const double t1 = __shfl_down_sync(FULL, suf, off), t2 = __shfl_down_sync(FULL, wsuf, off);
      if (lane + off < 32) { suf += t1; wsuf += t2; }
    }
    double pre = o * ldexp(1.0, lane + 1);          // count bound of octaves <= lane
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const double t = __shfl_up_sync(FULL, pre, off);
      if (lane >= off) pre += t;
    }
    const double Se = __shfl_sync(FULL, suf, 0), Ee = __shfl_sync(FULL, wsuf, 0);
    const double below = __shfl_down_sync(FULL, suf, 1), wbelow = __shfl_down_sync(FULL, wsuf, 1);
    const double blw = lane < 31 ? below : 0.0, wblw = lane < 31 ? wbelow : 0.0;   // octaves > lane
    K0Oct O;
    O.Se = Se;
    O.Ee = Ee;
    O.Th = rc.thr * Se;
    O.rnd = 2.0 * ((4.0 * V + 16.0) * U53 * Se);
    const double es = est_err(Se, Ee, rc.m_y, 33, V);
    O.bc = -1;
    O.cum = 0.0;
    O.Eb = 0.0;
    int bl = -1;
    if (rc.thr > 0.0) {
      // crossing octave: suffix sum (from the deep end) first exceeds Th
      const unsigned cr = __ballot_sync(FULL, lane <= NOCT && suf > O.Th);
      O.bc = cr ? 31 - __clz(cr) : -1;
      if (O.bc < 0 || O.bc == NOCT) return ROW_GENERAL;
      O.cum = __shfl_sync(FULL, blw, O.bc);
      O.Eb = __shfl_sync(FULL, wblw, O.bc);
      // the list: octaves 0..bl, bl >= bc the first whose tail is clearly below Th
      const bool okl = lane >= O.bc && lane < NOCT &&
                       blw + 2.0 * est_err(blw, wblw, rc.m_y, 33, V) + rc.thr * es + O.rnd < O.Th;
      const unsigned lb = __ballot_sync(FULL, okl);
      bl = lb ? __ffs(lb) - 1 : -1;
      if (bl >= 0) {
        // go deeper while the list stays short, until the tail is below Th/64:
        // the list kernel's decision band (which scales with the tail) then
        // rarely reaches the crossing element
        const unsigned small = __ballot_sync(FULL, lane >= bl && lane < NOCT && blw <= O.Th * 0.015625);
        const unsigned fits = __ballot_sync(FULL, lane >= bl && lane < NOCT && pre <= 0.5 * LCAP);
        const int bt = small ? __ffs(small) - 1 : NOCT - 1;
        const int bf = fits ? 31 - __clz(fits) : bl;
        bl = max(bl, min(bt, bf));
      }
    }
    const double nb = bl >= 0 ? __shfl_sync(FULL, pre, bl) : 1e300;
    if (bl >= 0 && !forced && nb <= 2.0 * LCAP) {
      unsigned long long mask = 0ull;
      float xmx = -INFINITY;
#pragma unroll
      for (int j = 0; j < OWN; ++j) {
        if ((est_rank(__expf(dest(rc, x[j]))) >> 8) <= bl) mask |= 1ull << j;
        else xmx = fmaxf(xmx, x[j]);
      }
      int ng;
      const int wpos = block_exscan_i32(__popcll(mask), S.redi, &ng);
      if (ng <= LCAP) {
        write_keys(a.lkeys + (size_t)row * LCAP, rc, x, mask, wpos);
        const float xm = block_reduce(xmx, MaxF(), S.redf);
        const double tl = __shfl_sync(FULL, blw, bl), et = __shfl_sync(FULL, wblw, bl);
        if (tid == 0) {
          RowJob& J = a.jobs[row];
          fill_job(J, rc, JOB_K0, ng, 0);
          queue_long_list(a, row, ng);
          J.tail = tl;
          J.tail_err = est_err(tl, et, rc.m_y, 33, V);
          J.ykex = xm > -INFINITY ? fkey(yex(rc, xm)) : 0u;
        }
        if (a.out_logits) write_row_regs(a, rc, x, true);
        return ROW_DONE;
      }
    }
    csync();                                        // the bins are read before the area is reused
    // the copy keeps x itself in registers: only xc's address reaches the call
    float xc[OWN];
#pragma unroll
    for (int j = 0; j < OWN; ++j) xc[j] = x[j];
    return k0_big(a, rc, xc, work, S, forced, O);
  }

  // ---- top-k rows: candidates >= the maxima threshold form the list ----
  // warps whose 32 lanes all own row positions: their maxima seed the list
  const int wfull = min(NWARP, ((V + shift + OWN - 1) / OWN) >> 5);
  if (wfull == 0 || k > wfull * (two ? 64 : 32)) return ROW_GENERAL;
  const int kw = (k + wfull - 1) / wfull;
  const unsigned wthr = two ? warp_kth_largest64(fkey(tm), fkey(t2), kw) : warp_kth_largest32(fkey(tm), kw);
  // each full warp has >= kw elements >= its wthr, so >= k elements are >= tau
  if (lane == 0) S.redu[warp] = wthr;
  csync();
  unsigned tkey = S.redu[0];
  for (int w = 1; w < wfull; ++w) tkey = S.redu[w] < tkey ? S.redu[w] : tkey;
  const float tau = fkey_inv(tkey);
  // fl(x/T) merges x only with values at most |x| 2^-23 below it: lowering tau
  // by 2^-18 relative (+ 2^-18 absolute) keeps every x tied with tau after /T
  const float tau_lo = tau - (fabsf(tau) + 1.0f) * 3.814697265625e-06f;
  if (!(tau_lo > -INFINITY)) return ROW_GENERAL;
  unsigned long long mask = 0ull;
#pragma unroll
  for (int j = 0; j < OWN; ++j)
    if (x[j] >= tau_lo) mask |= 1ull << j;
  int ng;
  const int wpos = block_exscan_i32(__popcll(mask), S.redi, &ng);   // its barriers also order S.redu
  if (ng > LCAP) return ROW_GENERAL;
  write_keys(a.lkeys + (size_t)row * LCAP, rc, x, mask, wpos);
  if (tid == 0) {
    RowJob& J = a.jobs[row];
    fill_job(J, rc, JOB_TOPK, ng, k);
    queue_long_list(a, row, ng);
    J.tail = 0.0;
    J.tail_err = 0.0;
    J.ykex = 0u;
  }
  if (a.out_logits) write_row_regs(a, rc, x, true);
  return ROW_DONE;
}

// ---------------------------------------------------------------------------
// The row kernel: rows blockIdx.x, +gridDim.x, ... of the chunk. Each row is
// staged into shared memory by one bulk-async copy (its <= 3-element unaligned
// head and tail by plain loads held in registers), penalised there, and read
// into registers; the buffer then takes the next row's copy at once (after
// the work of a row without top-k, which uses it as scratch). The next row's
// metadata arrives by cp.async.
// ---------------------------------------------------------------------------
struct Staged {
  int shift, body;           // body: bulk-copied elements (0: nothing in flight)
  int hpos;                  // buffer position of this thread's plain-loaded element (-1: none)
  float hval;
};
__device__ __forceinline__ Staged stage_row(const float* g, int V, float* rowbuf, unsigned long long* bar) {
  const unsigned long long ga = (unsigned long long)g;
  int head = (int)(((16u - (unsigned)(ga & 15ull)) & 15u) >> 2);
  if (head > V) head = V;
  const int body = ((V - head) >> 2) << 2;
  const int shift = (4 - head) & 3;
  const int tid = threadIdx.x;
  if (tid == 0 && body > 0) {
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(bar, (unsigned)body * 4u);
    bulk_g2s(rowbuf + shift + head, g + head, (unsigned)body * 4u, bar);
  }
  Staged st{shift, body, -1, 0.0f};
  int i = -1;
  if (tid < 4) i = tid < head ? tid : -1;
  else if (tid < 8) i = head + body + (tid - 4) < V ? head + body + (tid - 4) : -1;
  if (i >= 0) {
    st.hpos = shift + i;
    st.hval = __ldcs(g + i);
  }
  return st;
}

__global__ void __launch_bounds__(NT, 2) row_kernel(Args a) {
  extern __shared__ __align__(16) unsigned char dsm[];   // the staged row, then scratch
  __shared__ Shared S;
  __shared__ unsigned bm[(F_MAXV + 31) / 32 + 4];        // penalty de-duplication bitmap
  __shared__ MetaSlot meta[2];
  float* rowbuf = reinterpret_cast<float*>(dsm);
  const int V = a.V;
  const int tid = threadIdx.x;
  const int G = gridDim.x;
  const int nbm = (V + 31) / 32;

  if (tid == 0) mbar_init(&S.bar, 1);
  int act_pend = 1;
  auto issue_meta = [&](int r, MetaSlot& ms) {
    if (r >= a.B) return;
    const char* prm = reinterpret_cast<const char*>(a.params + (long long)r * a.params_stride);
    if (tid < 3) cp_async8(reinterpret_cast<char*>(&ms.P) + 8 * tid, prm + 8 * tid);
    else if (tid == 3) { if (a.hist_off) cp_async8(&ms.off0, a.hist_off + r); else ms.off0 = 0; }
    else if (tid == 4) { if (a.hist_off) cp_async8(&ms.off1, a.hist_off + r + 1); else ms.off1 = 0; }
    else if (tid == 5) cp_async8(&ms.rng, a.rng + r);
    else if (tid == 6) act_pend = a.active ? (int)a.active[r] : 1;
  };
  // rows are handed out dynamically (the first G statically): a CTA that
  // meets slow rows takes fewer of them
  unsigned* row_ctr = a.defer_cnt + 2;
  const int r0 = blockIdx.x;
  if (tid == 0) S.nrow[0] = G + (int)atomicAdd(row_ctr, 1u);
  issue_meta(r0, meta[0]);
  cp_async_commit();
  if (tid == 6 && r0 < a.B) meta[0].active = act_pend;
  cp_async_wait<0>();
  csync();
  unsigned phase = 0;
  Staged sg{0, 0, -1, 0.0f};
  if (r0 < a.B && meta[0].active) sg = stage_row(a.logits + (long long)r0 * a.ld, V, rowbuf, &S.bar);

  int j = 0;
  for (int row = r0; row < a.B; ++j) {
    const MetaSlot& cur = meta[j & 1];
    MetaSlot& nxt = meta[(j + 1) & 1];
    const int next = S.nrow[j & 1];
    issue_meta(next, nxt);
    cp_async_commit();
    if (tid == 6 && next < a.B) nxt.active = act_pend;
    bool staged_next = false;
    if (cur.active) {
      const c4s_row_params P = cur.P;
      const bool pen = a.hist_off && P.repetition_penalty != 1.0f;
      long long h0 = 0, h1 = 0;
      if (pen) {
        h0 = cur.off0;
        h1 = cur.off1;
        if (h0 < 0 || h1 < h0 || h1 > a.hist_total) {
          if (tid == 0) atomicOr(a.errflags, C4S_DEVERR_HIST_RANGE);
          h0 = h1 = 0;
        }
        for (int w = tid; w < nbm; w += NT) bm[w] = 0u;
      }
      int hid[8];
      hist_prefetch(a, h0, h1, hid);
      // the staged row (bounded wait), its plain-loaded edges, the penalty
      if (tid == 0) {
        bool ok = true;
        if (sg.body > 0) ok = mbar_wait_bounded(&S.bar, phase);
        S.abort_row = ok ? 0 : 1;
        if (!ok) atomicOr(a.errflags, C4S_DEVERR_TIMEOUT);
      }
      if (sg.body > 0) phase ^= 1u;
      if (sg.hpos >= 0) rowbuf[sg.hpos] = sg.hval;
      csync();
      if (S.abort_row) {
        if (tid == 0) mbar_wait_bounded(&S.bar, phase ^ 1u);   // let the copy drain (bounded)
        break;
      }
      float* srow = rowbuf + sg.shift;
      if (pen) penalty_apply(a, srow, V, bm, P.repetition_penalty, hid, h0, h1);
      float x[OWN];
      load_block(rowbuf, sg.shift, V, x);
      const int shift = sg.shift;
      csync();                                     // every thread has its elements
      // rows without top-k use the buffer as scratch: stage the next row after them
      const bool scratch = !P.greedy && !(P.top_k > 0 && P.top_k < V);
      if (!scratch && next < a.B && nxt.active) {
        sg = stage_row(a.logits + (long long)next * a.ld, V, rowbuf, &S.bar);
        staged_next = true;
      }
      if (row_body(a, row, cur, x, shift, dsm, S) == ROW_GENERAL) {
        csync();
        if (tid == 0) {
          a.jobs[row].kind = JOB_DEFER;
          defer_row(a, row);
        }
      }
      if (scratch) csync();                        // scratch released
    } else if (tid == 0) {
      a.out_ids[row] = -1;
      a.jobs[row].kind = JOB_NONE;
    }
    if (tid == 0) S.nrow[(j + 1) & 1] = next < a.B ? G + (int)atomicAdd(row_ctr, 1u) : a.B;   // the row after next
    cp_async_wait<0>();
    csync();                                       // next metadata visible
    if (!staged_next) {
      sg = Staged{0, 0, -1, 0.0f};
      if (next < a.B && nxt.active) sg = stage_row(a.logits + (long long)next * a.ld, V, rowbuf, &S.bar);
    }
    row = next;
  }
}

// ---------------------------------------------------------------------------
// The general path for the rows the row and list kernels handed back; the
// last CTA to finish clears the hand-back list for the next launch sequence.
// ---------------------------------------------------------------------------
// A no-top-k row whose top-p decision fell inside the band of its estimated
// tail: the exact tail mass (sum of exp((double)(y - m_y)) over the elements
// below the list, re-associated; its rounding is inside the list's double-sum
// band) replaces the estimate and the list job runs again on warp 0.
// Returns 1 if the row is finished, 0 if it needs the general path, -1 if the
// staging wait gave up.
__device__ __noinline__ int refine_k0(const Args& a, int row, float* rowbuf, unsigned* bitmap, Shared& S,
                                      LRed& R, unsigned long long* hist, unsigned* vk_area, double* pv_area,
                                      unsigned& phase) {
  const int V = a.V;
  const int tid = threadIdx.x;
  const c4s_row_params P = a.params[(long long)row * a.params_stride];
  const Stage sg = stage_issue(a.logits + (long long)row * a.ld, V, rowbuf, &S.bar);
  const bool pen = a.hist_off && P.repetition_penalty != 1.0f;
  long long h0, h1;
  hist_window(a, row, pen, h0, h1);
  int hid[8];
  hist_prefetch(a, h0, h1, hid);
  if (pen)
    for (int w = tid; w < (V + 31) / 32; w += NT) bitmap[w] = 0u;
  if (!stage_wait(a, sg, &S.bar, phase, S)) return -1;
  float* srow = rowbuf + sg.shift;
  if (pen) penalty_apply(a, srow, V, bitmap, P.repetition_penalty, hid, h0, h1);
  RowJob& J = a.jobs[row];
  const float T = P.temperature;
  const bool do_t = !(T == 1.0f || T <= 0.0f);
  const float rT = do_t ? __frcp_rn(T) : 1.0f;
  const unsigned ykex = J.ykex;
  const float m_y = J.m_y;
  double t = 0.0;
  for (int i = tid; i < V; i += NT) {
    const float y = do_t ? div_rn(srow[i], T, rT) : srow[i];
    if (fkey(y) <= ykex) t += prob(y, m_y);
  }
  double tail;
  block_exscan_f64(t, S.redd, &tail);
  if (tid == 0) {
    J.tail = tail;
    J.tail_err = 0.0;
  }
  csync();
  // the staged list: value keys in the sort-key area (2 LIST_CAP entries), its
  // probabilities in the row buffer (free once the tail is summed) or in the
  // probability area (LIST_CAP entries)
  const int n = J.n;
  double* pvs = nullptr;
  if ((size_t)n * 8 <= align_up((size_t)(V + 4) * 4, 16)) pvs = reinterpret_cast<double*>(rowbuf);
  else if (n <= LIST_CAP) pvs = pv_area;
  if (pvs == nullptr || n > 2 * LIST_CAP) return 0;
  const size_t o = (size_t)row * LCAP;
  const bool done = list_job<true>(a, row, J, a.lkeys + o, a.lsb + o, vk_area, pvs, hist, true, R);
  csync();
  return done ? 1 : 0;
}

__global__ void __launch_bounds__(NT, 4) defer_kernel(Args a) {
  extern __shared__ __align__(16) unsigned char dsm[];
  __shared__ Shared S;
  __shared__ LRed R;
  __shared__ unsigned long long lhist[256];
  const Layout L = layout_for(a.V);
  float* rowbuf = reinterpret_cast<float*>(dsm + L.row);
  unsigned* bitmap = reinterpret_cast<unsigned*>(dsm + L.bitmap);
  unsigned* cnt = reinterpret_cast<unsigned*>(dsm + L.cnt);
  unsigned long long* mass = reinterpret_cast<unsigned long long*>(dsm + L.mass);
  unsigned long long* lkey = reinterpret_cast<unsigned long long*>(dsm + L.key);
  double* pv = reinterpret_cast<double*>(dsm + L.pv);
  if (threadIdx.x == 0) mbar_init(&S.bar, 1);
  csync();
  unsigned phase = 0;
  const unsigned n = *reinterpret_cast<volatile unsigned*>(a.defer_cnt);
  for (unsigned t = blockIdx.x; t < n; t += gridDim.x) {
    const int row = a.defer_rows[t];
    if (a.jobs[row].kind == JOB_K0 && a.jobs[row].status == RES_REFINE) {
      const int r = refine_k0(a, row, rowbuf, bitmap, S, R, lhist, reinterpret_cast<unsigned*>(lkey), pv, phase);
      if (r < 0) break;
      if (r > 0) continue;
    }
    if (!general_row(a, row, rowbuf, bitmap, cnt, mass, lkey, pv, S, phase)) break;
  }
  csync();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&a.defer_cnt[1], 1u) == gridDim.x - 1) {
      a.defer_cnt[0] = 0u;
      a.defer_cnt[1] = 0u;
      a.defer_cnt[2] = 0u;                          // the row kernel's row counter
      a.defer_cnt[3] = 0u;                          // long lists queued for the list kernel
      a.defer_cnt[4] = 0u;                          //   and the list kernel's ticket
    }
  }
}

// ---------------------------------------------------------------------------
// Processed logits of list rows: the row kernel wrote the tempered values;
// mask what the list kernel's top-k threshold and K* remove.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NT) mask_kernel(Args a) {
  const int row = blockIdx.x;
  if (row >= a.B) return;
  const RowJob& J = a.jobs[row];
  if ((J.kind != JOB_TOPK && J.kind != JOB_K0) || J.status != RES_DONE) return;
  const unsigned tk = J.thresh_key;
  const unsigned long long kst = J.kstar;
  float* o = a.out_logits + (long long)row * a.out_ld;
  for (int i = threadIdx.x; i < a.V; i += NT) {
    const float y = o[i];
    if (fkey(y) < tk || (y > -INFINITY && ckey(y, i) < kst)) o[i] = -INFINITY;
  }
}

}  // namespace c4s
