// c4s_fast.cuh -- the fast path of the fused sampling step (MODE_SAMPLE, rows
// of up to F_MAXV logits): per chunk of at most K_CHUNK rows,
//
//   row_kernel (c4s_row.cuh): penalty, row maximum, and per row either the
//     greedy id or a candidate list in index order with a job record
//     (RowJob): top-k rows get the elements above a threshold that keeps at
//     least k of them; rows without top-k get the octaves of an error-bounded
//     probability estimate down to the top-p crossing plus an estimated tail.
//     List entries are ckey(x, i) of the penalised, untempered values.
//   list_kernel: per list (one warp for up to LW_CAP entries, else a whole
//     CTA from a queue): tempered value keys and exact double probabilities
//     staged in shared memory, the k-th largest value and the top-p crossing
//     by radix searches, then the draw by an index-order prefix
//     (sampling.cpp:30-71, text2semantic.cpp:150-165).
//   defer_kernel: rows the others hand back -- first the exact-tail
//     refinement of undecided rows without top-k, then the general path
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
#include "c4s_exp.cuh"

namespace c4s {

constexpr int F_MAXV = 9212;              // widest row the fast path takes
constexpr int LCAP = 9216;                // candidates per list (>= F_MAXV: a list can hold a whole row)
constexpr int LIST_DEEP = 1024;           // rows without top-k: lists go deeper only up to this length
constexpr int K_CHUNK = 4096;             // largest rows per launch sequence (list storage)
constexpr int NOCT = 30;                  // octaves of the estimate (<= 31: one warp lane each); bin NOCT = the rest
constexpr int LIST_WARPS = 8;             // list kernel: rows (warps) per CTA
constexpr int LW_CAP = 1024;              // list kernel: longest list one warp takes
constexpr int RQ_CAP = 16;                // list kernel: rows of one CTA waiting for an exact tail
constexpr int LIST_CLASSES = 6;           // list queues: long (CTA), then warp lists by size, longest first
constexpr int ROW_CLASSES = 4;            // cost classes of the row kernel's order
constexpr int ORD_CNT = 3 + 2 * LIST_CLASSES;   // first of their counters in defer_cnt
constexpr int NCNT = 20;                  // slots of the per-launch counters (defer_cnt)
static_assert(ORD_CNT + ROW_CLASSES <= NCNT, "the queue and order counters fit");

enum { JOB_NONE = 0, JOB_TOPK = 1, JOB_K0 = 2, JOB_DEFER = 3 };
enum { RES_DONE = 0, RES_DEFER = 1, RES_REFINE = 2 };

// Per-row job record: written by the row kernel, finished by the list kernel.
struct __align__(16) RowJob {
  int kind, n, k, status;
  float m_y;                 // row maximum after temperature
  unsigned ykex;             // JOB_K0: key of the largest value below the list (0: none)
  unsigned thresh_key;       // result: top-k threshold key (0: none)
  float T;                   // temperature (1: none); the list holds untempered values
  double thr, u;             // 1 - top_p; uniform of the draw
  double tail, tail_err;     // JOB_K0: estimated mass below the list and its error bound
  unsigned long long u53, xs;
  unsigned long long kstar;  // result: keys below K* are removed by top-p
  unsigned vcross;           // JOB_K0 handed to a refinement: value key of the crossing group
                             // the first pass found (0: none); the refinement's search starts there
  unsigned pad2;
};

// Per-row metadata, fetched asynchronously one row ahead.
struct __align__(16) MetaSlot {
  c4s_row_params P;          // 24 B
  long long off0, off1;      // history window [off0, off1)
  unsigned long long rng;    // xorshift64 state before this step
  int active;
  int hlen;                  // history window length (windowed histories; off1 unused)
};

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

// |d| = |y - m_y| of an element in octave b is below (b+1) ln 2 (up to the
// estimate's own tiny error); the open octave NOCT holds everything down to
// the clamp at -200.
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

// Reduction scratch of a list job run by a whole CTA, and exp_tail's table
// (staged into shared memory once per launch by every kernel that runs list jobs).
struct LRed {
  double tab[64];
  double d[NWARP];
  double d3[NWARP][3];
  unsigned long long q3[NWARP][3];
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
  // Three sums at once (one pair of barriers in a CTA).
  __device__ static void sum3(double& x, double& y, double& z, LRed& R) {
    x = warp_sum_d(x);
    y = warp_sum_d(y);
    z = warp_sum_d(z);
    if (!CTA) return;
    if ((threadIdx.x & 31) == 0) {
      R.d3[threadIdx.x >> 5][0] = x;
      R.d3[threadIdx.x >> 5][1] = y;
      R.d3[threadIdx.x >> 5][2] = z;
    }
    csync();
    x = y = z = 0.0;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) { x += R.d3[w][0]; y += R.d3[w][1]; z += R.d3[w][2]; }
    csync();
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

// Ascending bitonic sort of 32*SL keys held SL per lane (lane l: positions
// SL*l .. SL*l+SL-1), in registers: within-lane stages by compare-exchange,
// the others by shuffles. Whole warp calls.
template <int SL, typename T>
__device__ __forceinline__ void warp_sort_regs(T (&v)[SL]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 32 * SL; k <<= 1) {
#pragma unroll
    for (int jj = k >> 1; jj > 0; jj >>= 1) {
      if (jj < SL) {
#pragma unroll
        for (int j = 0; j < SL; ++j) {
          const int p = j ^ jj;
          if (p > j) {
            const bool up = ((SL * lane + j) & k) == 0;
            const T lo = v[j] < v[p] ? v[j] : v[p], hi = v[j] < v[p] ? v[p] : v[j];
            v[j] = up ? lo : hi;
            v[p] = up ? hi : lo;
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < SL; ++j) {
          const T o = __shfl_xor_sync(FULL, v[j], jj / SL);
          const int i = SL * lane + j;
          const bool keep_min = ((i & jj) == 0) == ((i & k) == 0);
          v[j] = keep_min ? (o < v[j] ? o : v[j]) : (o < v[j] ? v[j] : o);
        }
      }
    }
  }
}

// The k-th largest of n <= 32*SL value keys staged in vk (one warp).
template <int SL>
__device__ __forceinline__ unsigned warp_kth_sorted(const unsigned* vk, int n, int k) {
  const int lane = threadIdx.x & 31;
  unsigned v[SL];
#pragma unroll
  for (int j = 0; j < SL; ++j) {
    const int e = SL * lane + j;
    v[j] = e < n ? vk[e] : 0u;                     // padding sorts first
  }
  warp_sort_regs<SL>(v);
  const int pos = 32 * SL - k;
  unsigned r = 0u;
#pragma unroll
  for (int j = 0; j < SL; ++j) r = (pos % SL == j) ? v[j] : r;
  return __shfl_sync(FULL, r, pos / SL);
}

// Top-p crossing of at most 32*SL survivors (vk >= tk) by one warp: their
// keys (value << 32 | position; positions are in index order, so this is the
// canonical (value, index) order) are gathered into `buf`, sorted in
// registers, and the first sorted position whose running mass from the low
// end (starting at `tail`) exceeds Th is the crossing. Returns false if none;
// else its list position and the running masses before and at it.
template <int SL>
__device__ __forceinline__ bool warp_sorted_crossing(const unsigned* vk, const double* pv, int n, unsigned tk, int ns,
                                                     double tail, double Th, unsigned long long* buf, int* pos,
                                                     double* before, double* cur) {
  const int lane = threadIdx.x & 31;
  int base = 0;
  for (int e0 = 0; e0 < n; e0 += 32) {
    const int e = e0 + lane;
    const bool sv = e < n && vk[e] >= tk;
    const unsigned bal = __ballot_sync(FULL, sv);
    if (sv) buf[base + __popc(bal & ((1u << lane) - 1u))] = ((unsigned long long)vk[e] << 32) | (unsigned)e;
    base += __popc(bal);
  }
  for (int i = ns + lane; i < 32 * SL; i += 32) buf[i] = KEY_MAX;
  __syncwarp();
  unsigned long long v[SL];
#pragma unroll
  for (int j = 0; j < SL; ++j) v[j] = buf[SL * lane + j];
  __syncwarp();
  warp_sort_regs<SL>(v);
  double p[SL], s = 0.0;
#pragma unroll
  for (int j = 0; j < SL; ++j) {
    p[j] = v[j] != KEY_MAX ? pv[(int)(v[j] & 0xffffffffull)] : 0.0;
    s += p[j];
  }
  double incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(FULL, incl, o);
    if (lane >= o) incl += y;
  }
  double run = tail + incl - s, bf = 0.0, cu = 0.0;
  unsigned long long kx = 0ull;
  bool hit = false;
#pragma unroll
  for (int j = 0; j < SL; ++j) {
    const double nx = run + p[j];
    if (!hit && nx > Th) { hit = true; bf = run; cu = nx; kx = v[j]; }
    run = nx;
  }
  const unsigned cb = __ballot_sync(FULL, hit);
  if (!cb) return false;
  const int L = __ffs(cb) - 1;
  *pos = (int)(__shfl_sync(FULL, kx, L) & 0xffffffffull);
  *before = __shfl_sync(FULL, bf, L);
  *cur = __shfl_sync(FULL, cu, L);
  return true;
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

// Fixed-point masses of the searches: p (<= 1) in units of 2^-48, truncated
// (the sums of up to LCAP of them stay below 2^62). Integer sums have none of
// the long dependent latency of double adds; the error, below one unit per
// element, only moves the search, which the caller checks.
constexpr double MASS_Q = 0x1p48;
static_assert((double)LCAP * MASS_Q < 0x1p62, "fixed-point masses of a list cannot overflow");
__device__ __forceinline__ unsigned long long mass_q(double p) { return __double2ull_rz(p * MASS_Q); }

// The same search by a whole CTA (long lists), by bisection two bits a step:
// three thresholds summed per step and one pair of barriers per step (no
// atomics: on thousands of keys contended shared-memory adds cost more). Each
// thread keeps a mask of its entries (entry tid + k NT: bit k) whose keys lie
// in the interval still searched, [v, v + 2^(b+1)), and the mass of its
// entries below it: an entry below the interval adds its mass to every later
// threshold, one above it to none, so only the entries inside are visited
// (four at a time, their loads in flight together) and the sums are the same
// integers as over the whole list. Once at most 32 entries are left inside,
// one warp finishes the search on them (one entry per lane, no CTA barriers).
// `scratch`: 64 words of shared memory the caller does not need meanwhile.
__device__ __forceinline__ unsigned bisect_mass_cta(const unsigned* __restrict__ vk, const double* __restrict__ pv,
                                                    int n, unsigned prefix, int b0, double base, double Th, LRed& R,
                                                    unsigned long long* scratch) {
  static_assert((LCAP + NT - 1) / NT <= 64, "a thread's entries fit the mask");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  unsigned v = prefix;
  const double thq = (Th - base) * MASS_Q;          // the mass allowed below the crossing
  const int per = n > tid ? (n - tid + NT - 1) / NT : 0;
  unsigned long long act = per >= 64 ? ~0ull : ((1ull << per) - 1ull);
  unsigned long long below = 0ull;                  // this thread's mass of entries below v
  unsigned long long* h_q = scratch;                // [32] the warp stage's entries: fixed-point masses,
  unsigned* h_e = reinterpret_cast<unsigned*>(scratch + 32);   // [32] their positions,
  unsigned* h_n = reinterpret_cast<unsigned*>(scratch + 48);   // [0] their count, [1] the result
  unsigned long long* h_below = scratch + 49;       // the mass below them
  if (tid == 0) {
    h_n[0] = 0u;
    *h_below = 0ull;
  }
  for (int b = b0; b >= 0; b -= 2) {
    const int lo = b >= 1 ? b - 1 : 0;
    const unsigned c0 = v | (1u << lo), c1 = v | (2u << lo), c2 = v | (3u << lo);
    const unsigned long long end = (unsigned long long)v + (2ull << b);
    unsigned long long s0 = 0ull, s1 = 0ull, s2 = 0ull, keep = 0ull;
    for (unsigned long long m = act; m;) {
      int kk[4];
      bool ok[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        ok[u] = m != 0ull;
        kk[u] = ok[u] ? __ffsll((long long)m) - 1 : 0;
        if (ok[u]) m &= m - 1ull;
      }
      unsigned x[4];
      double p[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int e = tid + kk[u] * NT;
        x[u] = ok[u] ? vk[e] : 0u;
        p[u] = ok[u] ? pv[e] : 0.0;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (!ok[u] || (unsigned long long)x[u] >= end) continue;   // above the interval: in no later sum
        const unsigned long long q = mass_q(p[u]);
        if (x[u] < v) {                             // below it: in every later sum
          below += q;
          continue;
        }
        keep |= 1ull << kk[u];
        s0 += x[u] < c0 ? q : 0ull;
        s1 += x[u] < c1 ? q : 0ull;
        s2 += x[u] < c2 ? q : 0ull;
      }
    }
    act = keep;
    unsigned long long g0 = below + s0, g1 = below + s1, g2 = below + s2;
    int na = __popcll(keep);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      g0 += __shfl_xor_sync(FULL, g0, o);
      g1 += __shfl_xor_sync(FULL, g1, o);
      g2 += __shfl_xor_sync(FULL, g2, o);
    }
    na = __reduce_add_sync(FULL, na);
    if (lane == 0) {
      R.q3[warp][0] = g0;
      R.q3[warp][1] = g1;
      R.q3[warp][2] = g2;
      R.i[warp] = na;
    }
    csync();
    g0 = g1 = g2 = 0ull;
    na = 0;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) {
      g0 += R.q3[w][0];
      g1 += R.q3[w][1];
      g2 += R.q3[w][2];
      na += R.i[w];
    }
    csync();
    if (lo < b && (double)g2 <= thq) v = c2;
    else if (lo < b && (double)g1 <= thq) v = c1;
    else if ((double)g0 <= thq) v = c0;
    if (b >= 2 && na <= 32) {
      // the entries inside the old interval (the new one lies in it) to one
      // warp; the mass below v they do not cover in h_below
      for (unsigned long long m = keep; m; m &= m - 1ull) {
        const int e = tid + (__ffsll((long long)m) - 1) * NT;
        const unsigned slot = atomicAdd(&h_n[0], 1u);
        h_e[slot] = (unsigned)e;
        h_q[slot] = mass_q(pv[e]);
      }
      unsigned long long wb = below;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) wb += __shfl_xor_sync(FULL, wb, o);
      if (lane == 0 && wb != 0ull) atomicAdd(h_below, wb);
      csync();
      if (warp == 0) {
        const unsigned cnt = h_n[0];
        unsigned x = 0xffffffffu;
        unsigned long long q = 0ull;
        if ((unsigned)lane < cnt) {
          x = vk[h_e[lane]];
          q = h_q[lane];
        }
        const unsigned long long bw = *h_below;
        for (int b2 = b - 2; b2 >= 0; b2 -= 2) {
          // g(c) = mass below the entries + theirs below c: an entry under
          // v counts in every sum, one at or above the interval's end in none
          const int lo2 = b2 >= 1 ? b2 - 1 : 0;
          const unsigned d0 = v | (1u << lo2), d1 = v | (2u << lo2), d2 = v | (3u << lo2);
          unsigned long long w0 = x < d0 ? q : 0ull, w1 = x < d1 ? q : 0ull, w2 = x < d2 ? q : 0ull;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            w0 += __shfl_xor_sync(FULL, w0, o);
            w1 += __shfl_xor_sync(FULL, w1, o);
            w2 += __shfl_xor_sync(FULL, w2, o);
          }
          w0 += bw;
          w1 += bw;
          w2 += bw;
          if (lo2 < b2 && (double)w2 <= thq) v = d2;
          else if (lo2 < b2 && (double)w1 <= thq) v = d1;
          else if ((double)w0 <= thq) v = d0;
        }
        if (lane == 0) h_n[1] = v;
      }
      csync();
      v = h_n[1];
      csync();                                      // the scratch is free again
      return v;
    }
  }
  return v;
}

// Top-p search of a list job over the value keys that share `prefix` above
// bit b0: the largest key c whose mass below, base + G(c) (G(c) = sum of p
// over keys < c; removed candidates have p = 0), is <= Th -- the value of the
// crossing element -- found DB bits at a time from b0 down. A pass sums the
// masses of the keys that share the prefix found so far into 2^DB bins by
// their next digit (64-bit integer atomics in shared memory `hist`) and takes the
// largest digit whose mass below is <= Th. The bins hold fixed-point masses
// (mass_q); the caller checks the group the search ends on against its own
// double sums and their rounding band, as it checks any search. Whole group
// calls.
template <bool CTA, int DB>
__device__ __forceinline__ unsigned radix_mass(const unsigned* __restrict__ vk, const double* __restrict__ pv, int n,
                                               unsigned prefix, int b0, double base, double Th,
                                               unsigned long long* __restrict__ hist, LRed& R) {
  using G = LG<CTA>;
  constexpr int NB = 1 << DB, PL = NB / 32;
  const int lane = threadIdx.x & 31;
  unsigned v = prefix;
  const double thq = (Th - base) * MASS_Q;          // the mass allowed below the crossing
  unsigned long long below = 0ull;                  // fixed-point mass below the prefix's range
  for (int hi = b0; hi >= 0;) {
    const int w = hi + 1 < DB ? hi + 1 : DB;
    const int lo = hi - w + 1;
    const unsigned pmask = hi >= 31 ? 0u : ~((2u << hi) - 1u);
    const unsigned dmask = (1u << w) - 1u;          // the digit: bits lo..hi
    for (int i = G::rank(); i < NB; i += G::N) hist[i] = 0ull;
    G::sync();
    for (int e = G::rank(); e < n; e += G::N) {
      const unsigned x = vk[e];
      const unsigned long long q = mass_q(pv[e]);
      if ((x & pmask) == v && q != 0ull) atomicAdd(&hist[(x >> lo) & dmask], q);
    }
    G::sync();
    if (!CTA || threadIdx.x < 32) {
      unsigned long long c[PL], sl = 0ull;
#pragma unroll
      for (int j = 0; j < PL; ++j) { c[j] = hist[PL * lane + j]; sl += c[j]; }
      unsigned long long incl = sl;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(FULL, incl, o);
        if (lane >= o) incl += y;
      }
      // the bins whose mass below is within the budget are a prefix [0, D] of the digits
      unsigned long long run = below + (incl - sl), ex = below;
      int cnt = 0;
#pragma unroll
      for (int j = 0; j < PL; ++j) {
        if ((double)run <= thq) { ++cnt; ex = run; }
        run += c[j];
      }
      int d = __reduce_add_sync(FULL, cnt) - 1;    // bins above the digit's range are empty
      d = d < 0 ? 0 : d > (int)dmask ? (int)dmask : d;
      const unsigned long long exd = __shfl_sync(FULL, ex, d / PL);
      if (CTA) {
        if (threadIdx.x == 0) { R.e = d; R.q[0] = exd; }
      } else {
        v |= (unsigned)d << lo;
        below = exd;
      }
    }
    if (CTA) {
      csync();
      v |= (unsigned)R.e << lo;
      below = R.q[0];
      csync();
    }
    hi = lo - 1;
  }
  return v;
}

// From a value key c of the list, steps to the neighbouring value group
// (next survivor key below or above) until it reaches the group whose mass
// range [base + G(v), base + G(v) + M(v)) holds Th, G(v) being the mass of
// the survivors below v and M(v) that of the group v: the group the searches
// (radix_mass, bisect_mass_cta) end on. A refinement whose exact tail moved the crossing by little gets
// there in a pass or two; false after 8 steps or past either end of the list
// (the caller then searches). Rounding differences against the searches' sums
// are harmless: the caller's band check accepts only a crossing that every
// summation order agrees on.
template <bool CTA>
__device__ __forceinline__ bool step_to_crossing(const unsigned* __restrict__ vk, const double* __restrict__ pv, int n,
                                                 unsigned tk, double base, double Th, unsigned c, unsigned* out,
                                                 LRed& R) {
  using G = LG<CTA>;
  for (int it = 0; it < 8; ++it) {
    double gs = 0.0, mg = 0.0, z = 0.0;
    unsigned long long below = 0ull, above = ~0ull;   // below: key + 1 (0: none)
    for (int e = G::rank(); e < n; e += G::N) {
      const unsigned x = vk[e];
      if (x < tk) continue;                           // removed by top-k: no mass
      if (x < c) {
        gs += pv[e];
        below = (unsigned long long)x + 1ull > below ? (unsigned long long)x + 1ull : below;
      } else if (x == c) {
        mg += pv[e];
      } else {
        above = (unsigned long long)x < above ? (unsigned long long)x : above;
      }
    }
    G::sum3(gs, mg, z, R);
    below = G::qmax(below, R);
    above = G::qmin(above, R);
    gs += base;
    if (mg > 0.0 && gs <= Th && gs + mg > Th) {
      *out = c;
      return true;
    }
    if (gs > Th) {
      if (below == 0ull) return false;
      c = (unsigned)(below - 1ull);
    } else {
      if (above == ~0ull) return false;
      c = (unsigned)above;
    }
  }
  return false;
}

// One list job. keys: the candidates' penalised, untempered value keys
// (keys.val(e)) and indices (keys.idx(e)) in index order (list position =
// index order), from a global ckey list (GlobalKeys) or from the staged row
// (the fused kernel). The job
// stages the keys of their tempered values y = fl(x/T) into vk[] and their
// probabilities into pv[] (zero for candidates that top-k removes), both in
// shared memory, so that its passes stay on chip; ykey(e) = ckey(y, i);
// pvg / sb (global) serve the rare exact fallback. Run by one warp (CTA =
// false) or by the whole CTA (long lists). With `refine` (the general kernel,
// after replacing an estimated tail by the exact one) a row that cannot be
// decided is not handed back: the caller finishes it on the general path.
// With INL (the fused kernel) an undecided row is not queued either: J.status
// says whether it needs an exact tail (RES_REFINE) or the general path.
// Returns whether the row is finished.
// Candidate keys of a list in global memory: ckey(x, i) per position.
struct GlobalKeys {
  const unsigned long long* __restrict__ k;
  __device__ __forceinline__ unsigned val(int e) const { return (unsigned)(__ldcg(k + e) >> 32); }
  __device__ __forceinline__ unsigned idx(int e) const { return (unsigned)(k[e] & 0xffffffffull); }
};

template <bool CTA, bool INL = false, typename KS = GlobalKeys>
__device__ __forceinline__ bool list_job(const Args& a, int row, RowJob& J, const KS keys, unsigned long long* sb,
                                         unsigned* __restrict__ vk, double* __restrict__ pv,
                                         unsigned long long* __restrict__ hist, bool refine, LRed& R, int* rq) {
  using G = LG<CTA>;
  const int r0 = G::rank();
  constexpr int GN = G::N;
  const int n = J.n, V = a.V, k = J.k;
  const float m_y = J.m_y;
  const bool k0 = J.kind == JOB_K0;
  const bool forced = (a.debug & C4S_DEBUG_FORCE_BINS) != 0;
  // rq: the list kernel CTA's queue of rows that need an exact tail
  // (rq[0] = count, capacity RQ_CAP); elsewhere they go to the general kernel
  auto hand_back = [&](int st) {
    if (INL) {                                      // the caller reads J.status and finishes the row
      if (r0 == 0 && !refine) J.status = st;
      return;
    }
    if (r0 == 0 && !refine) {
      J.status = st;
      const int slot = (st == RES_REFINE && rq != nullptr) ? atomicAdd(&rq[0], 1) : RQ_CAP;
      if (slot < RQ_CAP) rq[1 + slot] = row;
      else defer_row(a, row);
    }
  };
  auto ykey = [&](int e) { return ((unsigned long long)vk[e] << 32) | keys.idx(e); };
  // stage the tempered value keys (sampling.cpp:16): eight loads in flight per member
  const float T = J.T;
  const bool do_t = T != 1.0f;
  const float rT = do_t ? __frcp_rn(T) : 1.0f;
  unsigned long long vmin = ~0ull, vmax = 0ull;
  unsigned long long redo = 0ull;
  static_assert((LCAP + NT - 1) / NT <= 64 && (LW_CAP + 31) / 32 <= 64, "a member's entries fit the redo mask");
  for (int e0 = r0; e0 < n; e0 += 8 * GN) {
    unsigned v[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int e = e0 + q * GN;
      v[q] = e < n ? keys.val(e) : 0u;
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int e = e0 + q * GN;
      if (e < n) {
        const float x = fkey_inv(v[q]);
        bool ok = true;
        const unsigned y = fkey(do_t ? div_rn_try(x, T, rT, ok) : x);
        if (ok) {
          vk[e] = y;
          vmin = y < vmin ? y : vmin;
          vmax = y > vmax ? y : vmax;
        } else {
          redo |= 1ull << ((e - r0) / GN);
        }
      }
    }
  }
  // quotients div_rn_try could not prove (bit j: entry r0 + j GN)
  for (; redo; redo &= redo - 1ull) {
    const int e = r0 + (__ffsll(redo) - 1) * GN;
    const unsigned y = fkey(div_call(fkey_inv(keys.val(e)), T));
    vk[e] = y;
    vmin = y < vmin ? y : vmin;
    vmax = y > vmax ? y : vmax;
  }
  vmin = G::qmin(vmin, R);
  vmax = G::qmax(vmax, R);
  G::sync();
  // no-top-k list: everything below it must be strictly smaller in value
  if (k0 && J.ykex >= vmin) { hand_back(RES_DEFER); return false; }

  // ---- top-k threshold: the k-th largest value key (sampling.cpp:30-40) ----
  unsigned tk = (unsigned)vmin;
  if (k > 0 && k < n && vmin != vmax) {
    const int b0 = 31 - __clz((unsigned)(vmin ^ vmax));
    const unsigned v = b0 >= 31 ? 0u : ((unsigned)vmax & ~((2u << b0) - 1u));
    if (!CTA && n <= 64) tk = warp_kth_sorted<2>(vk, n, k);
    else if (!CTA && n <= 128) tk = warp_kth_sorted<4>(vk, n, k);
    else if (!CTA && n <= 256) tk = warp_kth_sorted<8>(vk, n, k);
    else tk = radix_kth<CTA>(vk, n, v, b0, k, hist, R);
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
      // the reference's exp((double)(y - max)) within 2^-51 (Tang's exp_tail);
      // the bands below cover it, and the exact fallbacks use prob()
      p = exp_tail(__fsub_rn(fkey_inv(v), m_y), R.tab);
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
  const unsigned long long kmax = ykey((int)G::qmax(elast, R));   // the largest survivor key
  G::sync();

  // ---- top-p (sampling.cpp:42-71) ----
  const double thr = J.thr;
  const double tail = J.tail;
  const double St = tail + ps;
  unsigned long long kst = 0ull;
  bool exact_tp = false;
  // the debug flag sends every first-pass no-top-k list to a refinement once its crossing is found
  const bool force_ref = k0 && !refine && (a.debug & C4S_DEBUG_FORCE_REFINE) != 0;
  if (thr < 0.0) {
    kst = 0ull;                                       // p > 1: nothing removed
  } else if (thr == 0.0) {
    unsigned long long mk0 = KEY_MAX;                 // p == 1: only zero probabilities go
    for (int e = r0; e < n; e += GN)
      if (vk[e] >= tk && pv[e] > 0.0) mk0 = ykey(e) < mk0 ? ykey(e) : mk0;
    kst = G::qmin(mk0, R);
  } else if (!CTA && ns <= 128) {
    // few survivors: sort them in registers and find the crossing on a prefix
    // scan (the 128 keys' buffer is the 1 KB histogram area)
    const double Th = thr * St;
    int pos = 0;
    double before = 0.0, cur = 0.0;
    const bool hit = ns <= 64 ? warp_sorted_crossing<2>(vk, pv, n, tk, ns, tail, Th, hist, &pos, &before, &cur)
                              : warp_sorted_crossing<4>(vk, pv, n, tk, ns, tail, Th, hist, &pos, &before, &cur);
    if (hit) {
      const double bd = 2.0 * ((4.0 * (k0 ? V : ns) + 16.0) * U53 * St) + 2.0 * J.tail_err;
      kst = ykey(pos);
      exact_tp = !(before <= Th - bd && cur > Th + bd);
    } else {
      kst = KEY_MAX;                                  // no crossing: only the kept maximum
      exact_tp = true;
    }
    exact_tp = exact_tp || forced || force_ref;
  } else {
    const double Th = thr * St;
    // G(c) = tail + sum of p over value keys < c (removed candidates have p = 0);
    // the largest c with G(c) <= Th is the value of the crossing element
    const unsigned smin32 = (unsigned)smin, vmax32 = (unsigned)vmax;
    const int b0 = (smin32 == vmax32) ? -1 : 31 - __clz(smin32 ^ vmax32);
    unsigned v = b0 < 0 ? smin32 : (b0 >= 31 ? 0u : (vmax32 & ~((2u << b0) - 1u)));
    // a refinement starts from the first pass's crossing and bisects only if that fails
    const bool near = refine && J.vcross != 0u && step_to_crossing<CTA>(vk, pv, n, tk, tail, Th, J.vcross, &v, R);
    if (!near) {
      if constexpr (CTA) v = bisect_mass_cta(vk, pv, n, v, b0, tail, Th, R, hist);
      else v = radix_mass<false, 7>(vk, pv, n, v, b0, tail, Th, hist, R);
    }
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
      if (t == 1) {                                 // the group's first member: its least position
        unsigned long long me = ~0ull;
        for (int e = r0; e < n; e += GN)
          if (vk[e] == v) me = (unsigned long long)e < me ? (unsigned long long)e : me;
        es = (int)G::qmin(me, R);
      } else {
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
      }
      const double before = Gs + (double)(t - 1) * pg, cur = Gs + (double)t * pg;
      const double bd = 2.0 * ((4.0 * (k0 ? V : ns) + 16.0) * U53 * St) + 2.0 * J.tail_err;
      kst = ykey(es);
      exact_tp = !(before <= Th - bd && cur > Th + bd);
    } else {
      kst = KEY_MAX;                                  // no crossing: only the kept maximum
      exact_tp = true;
    }
    exact_tp = exact_tp || forced || force_ref;
  }
  if (exact_tp) {
    if (k0) {                                         // the tail is exact only after a refine
      if (!refine) {
        if (r0 == 0) J.vcross = kst != KEY_MAX ? (unsigned)(kst >> 32) : 0u;
        hand_back(RES_REFINE);
      }
      return false;
    }
    // the reference's sequential sums over the survivors in ascending order
    int base = 0;
    for (int e0 = 0; e0 < n; e0 += GN) {
      const int e = e0 + r0;
      const bool sv = e < n && vk[e] >= tk;
      int tot;
      const int pos = G::exscan_i(sv ? 1 : 0, R, &tot);
      if (sv) sb[base + pos] = ykey(e);
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
    return v >= tk && (v > kv || (v == kv && ykey(e) >= kst));
  };
  int tok = 0;
  if (J.u53 != 0ull) {
    // each member sums a contiguous range of positions; one exclusive scan of
    // those sums locates the member whose range the prefix crosses r in, and
    // that member scans its range
    const double u = J.u;
    const int L = (n + GN - 1) / GN;
    const int e_lo = min(r0 * L, n), e_hi = min(e_lo + L, n);
    double sm = 0.0;
    int cm = 0;
    for (int e = e_lo; e < e_hi; ++e)
      if (kept(e)) { sm += pv[e]; ++cm; }
    double s2;
    const double base = G::exscan_d(sm, R, &s2);
    const int nk = G::add(cm, R);
    const double r = u * s2;
    int fe = -1;
    double prev = 0.0, cur = 0.0;
    if (base < r && base + sm >= r) {
      double acc = base;
      for (int e = e_lo; e < e_hi; ++e) {
        if (kept(e)) {
          const double nx = acc + pv[e];
          if (nx >= r) { fe = e; prev = acc; cur = nx; break; }
          acc = nx;
        }
      }
    }
    const unsigned long long hit = G::qmin(fe >= 0 ? (unsigned long long)fe : ~0ull, R);
    int found = -1;
    if (hit != ~0ull) {
      found = (int)hit;
      G::bcast_2d(prev, cur, found / L, R);
    }
    const double bd2 = 2.0 * ((4.0 * nk + 16.0) * U53 * s2);
    if (!forced && found >= 0 && prev < r - bd2 && cur > r + bd2) {
      tok = (int)keys.idx(found);
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
            if (rr <= acc) { t = (int)keys.idx(e); break; }
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
// (staged value keys, probabilities) and 1 KB of scratch (a radix histogram of
// 256 counts, or the 128 keys of the sorted top-p crossing); once the warps
// are done, the same area holds one long list (up to LCAP) worked by the whole
// CTA. Sized so that two CTAs (16 warps) fit on an SM.
constexpr size_t LW_VK = 0, LW_PV = (size_t)LW_CAP * 4, LW_HIST = LW_PV + (size_t)LW_CAP * 8;
constexpr size_t LW_BYTES = LW_HIST + 128 * 8;            // per warp
static_assert(LW_BYTES - LW_HIST >= 256 * sizeof(unsigned), "radix histogram");
static_assert(LW_BYTES - LW_HIST >= 32 * 4 * sizeof(unsigned long long), "sorted-crossing keys");
static_assert(LW_BYTES - LW_HIST >= 128 * sizeof(unsigned long long), "a warp's top-p search bins");
constexpr size_t LB_VK = 0, LB_PV = (size_t)LCAP * 4, LB_HIST = LB_PV + (size_t)LCAP * 8;
constexpr size_t LIST_SMEM_W = (size_t)LIST_WARPS * LW_BYTES, LIST_SMEM_B = LB_HIST + 256 * 8;
constexpr size_t LIST_SMEM = LIST_SMEM_W > LIST_SMEM_B ? LIST_SMEM_W : LIST_SMEM_B;   // warps' areas / one long list

struct Staged {
  int shift, body;           // body: bulk-copied elements (0: nothing in flight)
  int hpos;                  // buffer position of this thread's plain-loaded element (-1: none)
  float hval;
};
// The 16-byte-aligned body of a row that stage_row copies, prefetched into L2
// one row ahead so that its DRAM reads overlap the current row's work.
__device__ __forceinline__ void prefetch_row(const float* g, int V) {
  const unsigned long long ga = (unsigned long long)g;
  int head = (int)(((16u - (unsigned)(ga & 15ull)) & 15u) >> 2);
  if (head > V) head = V;
  const int body = ((V - head) >> 2) << 2;
  if (body > 0) bulk_prefetch_l2(g + head, (unsigned)body * 4u);
}

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

__device__ const double EXP2_J64[64] = C4S_EXP2_J64_TABLE;   // exp_tail's table

// A row without top-k whose top-p crossing fell inside the band of its
// estimated tail, or whose list is long (a whole CTA's), in the list kernel
// (whole CTA): the exact tail mass (sum of
// exp((double)(y - m_y)) over every element below the list, each penalised
// and tempered as the reference does, re-associated: its rounding is inside
// the list's double-sum band; each term by exp_tail, within 2^-51 of the
// reference's, so tail_err = 2^-50 tail) replaces the estimate and the list job runs
// again, its top-p search starting from the first pass's crossing. A row
// still undecided goes to the general kernel. The raw row is staged by one
// bulk copy into the (still free) probability area, so the scan waits for one
// DRAM round trip; `lbar` is the CTA's mbarrier and lst[0] its phase, lst[1]
// set once a bounded wait has given up (later refinements then defer).
__device__ __noinline__ void refine_in_list(const Args& a, int row, unsigned* bm, unsigned* vk, double* pv,
                                            unsigned long long* hist, LRed& R, unsigned long long* lbar,
                                            unsigned* lst) {
  const int V = a.V, tid = threadIdx.x;
  RowJob& J = a.jobs[row];
  if (lst[1]) {
    if (tid == 0) defer_row(a, row);
    return;
  }
  const float* g = a.logits + (long long)row * a.ld;
  float* rowbuf = reinterpret_cast<float*>(pv);
  const Staged sg = stage_row(g, V, rowbuf, lbar);
  const c4s_row_params P = a.params[(long long)row * a.params_stride];
  bool pen = a.hist_off && P.repetition_penalty != 1.0f;
  long long h0 = 0, h1 = 0;
  if (pen) {
    h0 = a.hist_off[row];
    h1 = a.hist_len ? h0 + a.hist_len[row] : a.hist_off[row + 1];
    if (h0 < 0 || h1 < h0 || h1 > a.hist_total) pen = false;   // the row kernel flagged it
  }
  // history ids eight per thread at a time, the first batch in flight while the bitmap clears
  int hv[8];
  long long j0 = h0 + tid;
  auto load_ids = [&]() {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const long long j = j0 + (long long)q * NT;
      hv[q] = (pen && j < h1) ? a.hist[j] : -1;
    }
  };
  load_ids();
  for (int w = tid; w < (V + 31) / 32; w += NT) bm[w] = 0u;
  csync();
  if (pen) {
    for (;;) {
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if ((unsigned)hv[q] < (unsigned)V) atomicOr(&bm[hv[q] >> 5], 1u << (hv[q] & 31));
      j0 += 8LL * NT;
      if (j0 >= h1) break;
      load_ids();
    }
  }
  if (tid == 0 && sg.body > 0) {
    if (mbar_wait_bounded(lbar, lst[0])) {
      lst[0] ^= 1u;
    } else {
      lst[1] = 1u;
      atomicOr(a.errflags, C4S_DEVERR_TIMEOUT);
      mbar_wait_bounded(lbar, lst[0]);             // let the copy drain (bounded)
    }
  }
  if (sg.hpos >= 0) rowbuf[sg.hpos] = sg.hval;
  csync();
  if (lst[1]) {
    if (tid == 0) defer_row(a, row);
    return;
  }
  const float pp = P.repetition_penalty, rpen = __frcp_rn(pp);
  const float T = J.T;
  const bool do_t = T != 1.0f;
  const float rT = do_t ? __frcp_rn(T) : 1.0f;
  const unsigned ykex = J.ykex;
  const float m_y = J.m_y;
  const float* srow = rowbuf + sg.shift;
  // each term: penalised, tempered, its exp if it lies below the list; four
  // independent sums per thread keep four exp_tail chains in flight
  // (quotients div_rn_try cannot prove are redone after the loop: bit k of
  // `redo` = element tid + k NT)
  unsigned long long redo = 0ull;
  auto term = [&](int i, bool exact) -> double {
    float x = srow[i];
    bool ok = true, ok2 = true;
    if (pen && ((bm[i >> 5] >> (i & 31)) & 1u))
      x = (x < 0.0f) ? __fmul_rn(x, pp) : exact ? div_rn(x, pp, rpen) : div_rn_try(x, pp, rpen, ok);
    const float y = (do_t && x > -INFINITY) ? (exact ? div_rn(x, T, rT) : div_rn_try(x, T, rT, ok2)) : x;
    if (!(ok && ok2)) {
      redo |= 1ull << ((i - tid) / NT);
      return 0.0;
    }
    return (x > -INFINITY && fkey(y) <= ykex) ? exp_tail(__fsub_rn(y, m_y), R.tab) : 0.0;
  };
  double t0 = 0.0, t1 = 0.0, t2 = 0.0, t3 = 0.0;
  int i = tid;
  for (; i + 3 * NT < V; i += 4 * NT) {
    t0 += term(i, false);
    t1 += term(i + NT, false);
    t2 += term(i + 2 * NT, false);
    t3 += term(i + 3 * NT, false);
  }
  for (; i < V; i += NT) t0 += term(i, false);
  for (; redo; redo &= redo - 1ull) t0 += term(tid + (__ffsll(redo) - 1) * NT, true);
  const double tail = LG<true>::sum((t0 + t1) + (t2 + t3), R);
  if (tid == 0) {
    J.tail = tail;
    J.tail_err = ldexp(tail, -50);
    atomicAdd(&a.counters[C4S_CNT_EXACT_TAIL], 1ull);
  }
  csync();                                          // the row buffer is free again
  const size_t o = (size_t)row * LCAP;
  if (!list_job<true>(a, row, J, GlobalKeys{a.lkeys + o}, a.lsb + o, vk, pv, hist, true, R, nullptr) && tid == 0) {
    J.status = RES_DEFER;
    defer_row(a, row);
  }
}

// Persistent: first the long lists (one CTA each, so the longest work starts
// at once), then the other lists (one warp each) by size class, longest
// first, all from the queues the row kernel fills; between them each CTA
// refines the rows of its own that need an exact tail (the general kernel
// resets the queues).
__global__ void __launch_bounds__(32 * LIST_WARPS, 2) list_kernel(Args a) {
  static_assert(32 * LIST_WARPS == NT, "the list kernel's CTA barrier counts NT threads");
  extern __shared__ __align__(16) unsigned char lsm[];
  __shared__ LRed R;
  __shared__ int next;
  __shared__ int rq[1 + RQ_CAP];
  __shared__ unsigned bm[(F_MAXV + 31) / 32 + 1];
  __shared__ Args sa;                               // for refine_in_list (no local copy)
  __shared__ unsigned long long lbar;               // refinements' bulk row copies
  __shared__ unsigned lst[2];                       // its phase; set after a wait gave up
  if (threadIdx.x < 64) R.tab[threadIdx.x] = EXP2_J64[threadIdx.x];
  if (threadIdx.x == 0) {
    rq[0] = 0;
    sa = a;
    mbar_init(&lbar, 1);
    lst[0] = 0u;
    lst[1] = 0u;
  }
  grid_dep_launch();
  grid_dep_wait();                                 // the row kernel's jobs, lists and queues
  const unsigned nbig = *reinterpret_cast<volatile unsigned*>(&a.defer_cnt[3]);
  unsigned* bvk = reinterpret_cast<unsigned*>(lsm + LB_VK);
  double* bpv = reinterpret_cast<double*>(lsm + LB_PV);
  unsigned long long* bh = reinterpret_cast<unsigned long long*>(lsm + LB_HIST);
  // the CTA's queued refinements, then the next long list; false when none is left
  auto cta_work = [&]() -> bool {
    for (;;) {
      csync();                                      // the area is free
      const int nq = min(rq[0], RQ_CAP);
      if (nq > 0) {
        const int r = rq[nq];
        csync();
        if (threadIdx.x == 0) rq[0] = nq - 1;
        refine_in_list(sa, r, bm, bvk, bpv, bh, R, &lbar, lst);
        continue;
      }
      if (threadIdx.x == 0) {
        const unsigned t = *reinterpret_cast<volatile unsigned*>(&a.defer_cnt[4]);
        next = (int)(t < nbig ? atomicAdd(&a.defer_cnt[4], 1u) : t);
      }
      csync();
      const int t = next;
      if (t >= (int)nbig) return false;
      const int r = a.big_rows[t];
      const size_t o = (size_t)r * LCAP;
      // a long list of a row without top-k gets its exact tail first: its
      // one pass is then final (no refinement behind it on the critical path)
      if (a.jobs[r].kind == JOB_K0) refine_in_list(sa, r, bm, bvk, bpv, bh, R, &lbar, lst);
      else list_job<true>(a, r, a.jobs[r], GlobalKeys{a.lkeys + o}, a.lsb + o, bvk, bpv, bh, false, R, rq);
    }
  };
  cta_work();
  // the other lists, one warp each, by size class, longest first
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned char* wa = lsm + (size_t)w * LW_BYTES;
  for (int q = 1; q < LIST_CLASSES; ++q) {
    const unsigned nq = *reinterpret_cast<volatile unsigned*>(&a.defer_cnt[3 + 2 * q]);
    if (nq == 0u) continue;
    volatile unsigned* tq = &a.defer_cnt[4 + 2 * q];
    for (;;) {
      // a plain read first: thousands of warps finding a class empty would
      // otherwise queue on one contended atomic
      unsigned t = 0u;
      if (lane == 0) {
        t = *tq;
        if (t < nq) t = atomicAdd(&a.defer_cnt[4 + 2 * q], 1u);
      }
      t = __shfl_sync(FULL, t, 0);
      if (t >= nq) break;
      const int row = a.big_rows[(size_t)q * a.chunk + t];
      const size_t o = (size_t)row * LCAP;
      list_job<false>(a, row, a.jobs[row], GlobalKeys{a.lkeys + o}, a.lsb + o, reinterpret_cast<unsigned*>(wa + LW_VK),
                      reinterpret_cast<double*>(wa + LW_PV), reinterpret_cast<unsigned long long*>(wa + LW_HIST),
                      false, R, rq);
    }
  }
  cta_work();                                       // refinements found on the short lists
}

// ===========================================================================
// Row-kernel helpers (the row kernel itself is in c4s_row.cuh)
// ===========================================================================

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

// A tight lower bound tau on the k-th largest element of a row: at least k
// elements are >= tau, and few more. U holds each thread's largest element
// (and its second largest with `two`). The k-th largest value of U is
// located in a 256-bin histogram of the key distances d = fkey(m_x) -
// fkey(v) (bin 0: d = 0; then eight bins per octave of d), and tau is the
// smallest value of that bin's key range, so every U value in the bins up to
// it -- at least k of them -- is >= tau. Returns -inf if U holds fewer than k
// finite values. `bins` is 256 words of shared memory, res one word; every
// thread of the group (NTH threads, barrier `sync`) calls.
__device__ __forceinline__ int ubin(unsigned d) {
  if (d == 0u) return 0;
  const int e = 31 - __clz(d);
  const unsigned sub = e >= 3 ? (d >> (e - 3)) & 7u : (d << (3 - e)) & 7u;
  return min(255, 1 + 8 * e + (int)sub);
}
template <int NTH, typename Sync>
__device__ __forceinline__ float u_threshold(float tm, float t2, bool two, float m_x, int k, unsigned* bins,
                                             unsigned* res, Sync sync, bool zeroed = false) {
  const int tid = threadIdx.x;
  if (!zeroed) {                                   // else the caller cleared them behind an earlier barrier
    for (int i = tid; i < 256; i += NTH) bins[i] = 0u;
    sync();
  }
  const unsigned km = fkey(m_x);
  if (tm > -INFINITY) atomicAdd(&bins[ubin(km - fkey(tm))], 1u);
  if (two && t2 > -INFINITY) atomicAdd(&bins[ubin(km - fkey(t2))], 1u);
  sync();
  if (tid < 32) {
    unsigned c[8], sl = 0u;
#pragma unroll
    for (int j = 0; j < 8; ++j) { c[j] = bins[8 * tid + j]; sl += c[j]; }
    unsigned incl = sl;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned y = __shfl_up_sync(FULL, incl, o);
      if (tid >= o) incl += y;
    }
    const unsigned hit = __ballot_sync(FULL, incl >= (unsigned)k);
    unsigned tkey = fkey(-INFINITY);
    if (hit) {
      const int L = __ffs(hit) - 1;
      int bs = 0;
      if (tid == L) {
        unsigned run = incl - sl;
        bs = 8 * L + 7;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          run += c[j];
          if (run >= (unsigned)k) { bs = 8 * L + j; break; }
        }
      }
      bs = __shfl_sync(FULL, bs, L);
      // the largest distance in bin bs (ubin is monotone in d); the last bin
      // is open: every finite value
      unsigned dmax;
      if (bs == 0) {
        dmax = 0u;
      } else if (bs == 255) {
        dmax = km - fkey(-3.4028234663852886e38f);
      } else {
        const int e = (bs - 1) >> 3, sub = (bs - 1) & 7;
        if (e >= 3) {
          dmax = (1u << e) + ((unsigned)(sub + 1) << (e - 3)) - 1u;
        } else {
          dmax = 1u;
          for (unsigned d = 1u; d < 8u; ++d)
            if (ubin(d) <= bs) dmax = d;
        }
      }
      const unsigned lim = km - fkey(-3.4028234663852886e38f);   // tau stays finite
      tkey = km - (dmax < lim ? dmax : lim);
    }
    if (tid == 0) *res = tkey;
  }
  sync();
  return fkey_inv(*res);
}

// Header fields common to both list job kinds (thread 0).
__device__ __forceinline__ void fill_job(RowJob& J, const RowCtx& rc, int kind, int n, int k) {
  J.kind = kind;
  J.n = n;
  J.k = k;
  J.status = RES_DONE;
  J.m_y = rc.m_y;
  J.T = rc.do_t ? rc.T : 1.0f;
  J.thresh_key = 0u;
  J.thr = rc.thr;
  J.u = rc.u;
  J.u53 = rc.u53;
  J.xs = rc.xs;
  J.kstar = 0ull;
  J.vcross = 0u;
}

// A list longer than one list-kernel warp takes goes to the CTA-wide queue.
__device__ __forceinline__ void queue_long_list(const Args& a, int row, int n) {
  // classes: > LW_CAP, (512, 1024], (256, 512], (128, 256], (64, 128], <= 64
  const int q = n > LW_CAP ? 0 : n > 512 ? 1 : n > 256 ? 2 : n > 128 ? 3 : n > 64 ? 4 : 5;
  a.big_rows[(size_t)q * a.chunk + atomicAdd(&a.defer_cnt[3 + 2 * q], 1u)] = row;
}

enum { ROW_DONE = 0, ROW_GENERAL = 1 };

// ---------------------------------------------------------------------------
// The general path for the rows the row and list kernels handed back; the
// last CTA to finish clears the hand-back list for the next launch sequence.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NT, 4) defer_kernel(Args a) {
  extern __shared__ __align__(16) unsigned char dsm[];
  __shared__ Shared S;
  __shared__ Args sa;                               // for general_row (no local copy)
  const Layout L = layout_for(a.V);
  float* rowbuf = reinterpret_cast<float*>(dsm + L.row);
  unsigned* bitmap = reinterpret_cast<unsigned*>(dsm + L.bitmap);
  unsigned* cnt = reinterpret_cast<unsigned*>(dsm + L.cnt);
  unsigned long long* mass = reinterpret_cast<unsigned long long*>(dsm + L.mass);
  unsigned long long* lkey = reinterpret_cast<unsigned long long*>(dsm + L.key);
  double* pv = reinterpret_cast<double*>(dsm + L.pv);
  if (threadIdx.x == 0) {
    mbar_init(&S.bar, 1);
    sa = a;
  }
  csync();
  unsigned phase = 0;
  grid_dep_launch();
  grid_dep_wait();                                 // the rows the row and list kernels handed back
  const unsigned n = *reinterpret_cast<volatile unsigned*>(a.defer_cnt);
  for (unsigned t = blockIdx.x; t < n; t += gridDim.x) {
    const int row = a.defer_rows[t];
    if (!general_row(sa, row, rowbuf, bitmap, cnt, mass, lkey, pv, S, phase)) break;
  }
  csync();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&a.defer_cnt[1], 1u) == gridDim.x - 1) {
      a.defer_cnt[0] = 0u;
      a.defer_cnt[1] = 0u;
      a.defer_cnt[2] = 0u;                          // the row kernel's row counter
#pragma unroll
      for (int c = 3; c < ORD_CNT + ROW_CLASSES; ++c) a.defer_cnt[c] = 0u;   // list queues, row order
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
