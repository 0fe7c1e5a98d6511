// c4s_fused.cuh -- the fused sampling kernel (sm_100a): one launch per step.
//
// One persistent CTA of NT = 256 threads works one row at a time, start to
// finish, rows handed out dynamically (text2semantic.cpp:303-331 semantics;
// sampling.cpp:14-76 processors):
//
//   stage      the row into shared memory by one bulk-async copy (TMA engine,
//              bounded mbarrier wait), prefetched into L2 one row ahead; the
//              row's metadata (parameters, history window, xorshift64 state)
//              arrives one row ahead by cp.async;
//   penalty    in shared memory (sampling.cpp:19-28): every history id reads
//              its logit, a CTA barrier, then every id writes the penalised
//              value, so duplicates write the same value and need no
//              de-duplication (histories up to 8 ids per thread; longer ones
//              use a shared-memory bitmap);
//   greedy     the first index of the maximum (sampling.cpp:73-76);
//   sampled    a candidate list built from the staged row -- top-k rows: every
//              element >= a maxima threshold that keeps >= k of them; rows
//              without top-k: the octaves of an error-bounded probability
//              estimate down to the top-p crossing, the rest an estimated tail
//              with a proven bound -- held as element indices in shared
//              memory, and the list job (c4s_fast.cuh list_job: temperature,
//              top-k, top-p and the xorshift64 draw, exact outside proven
//              error bands) runs on it in place: on one warp for short lists,
//              on the CTA for long ones;
//   exact tail a row without top-k whose top-p crossing falls inside its
//              estimated tail's band gets the exact tail sum from the staged
//              row (no second read of the row) and its list job runs again;
//   general    anything else (non-finite maxima, |max/T| >= 2^18,
//              min_tokens_to_keep != 1, lists over FLC entries, crossings still
//              undecided) runs the general path (general_row) in the same CTA.
//
// Every row is finished inside its CTA: there is no list or hand-back kernel
// and no row waits for another, so a CTA working a long list does not hold
// up the other CTAs' streaming of rows, and a B = 1 step is one launch.
#pragma once

namespace c4s {

// Row buffer: warp w owns 16-byte slots [w seg, (w+1) seg), seg a multiple of
// 32 (lane l reads slots l, l+32, ... of it: conflict-free 16-byte loads in
// index order within a warp); positions outside the row hold -inf.
constexpr int F_SLOTS = (((F_MAXV + 3 + 3) / 4 + NWARP - 1) / NWARP + 31) / 32 * 32 * NWARP;
constexpr size_t F_ROW_BYTES = (size_t)F_SLOTS * 16;
// The list area after the row buffer: FLC entries of element index (u16),
// tempered value key (u32) and probability (f64), then 2 KB for the list
// job's histogram / sorted crossing keys (also the penalty bitmap of long
// histories). Before a list exists, the key and probability arrays hold the
// octave bins of rows without top-k and each warp's staged candidate
// positions.
constexpr int FLC = 1024;
constexpr size_t FL_LI = F_ROW_BYTES;
constexpr size_t FL_VK = FL_LI + (size_t)FLC * 2;
constexpr size_t FL_PV = FL_VK + (size_t)FLC * 4;
constexpr size_t FL_HIST = FL_PV + (size_t)FLC * 8;
constexpr size_t F_FAST_BYTES = FL_HIST + 2048;
constexpr int FHREP = 8;                           // replicas of each warp's octave bins
constexpr int FUSED_CNT = NCNT;                    // the fused kernel's two counters follow the split path's
constexpr int FUSED_MAX_ROWS = 256;                // batches up to this size take the fused kernel
constexpr int F_WSTRIDE = FHREP * 33;              // words of one warp's bins (rows of 33 words)
constexpr int F_STAGE_CAP = FHREP * 32 * 2;        // u16 positions a warp stages in its bins' words
constexpr int F_HIST_WORDS = 8 * NT;               // history ids a thread holds in registers: 8
static_assert(FL_VK % 16 == 0 && FL_PV % 16 == 0 && FL_HIST % 16 == 0, "aligned list arrays");
static_assert((size_t)NWARP * F_WSTRIDE * 4 <= (size_t)FLC * 12, "octave bins fit in the key/probability arrays");
static_assert(FLC <= LW_CAP && FLC <= LCAP, "a list the warp job takes fits its staging");
static_assert(((F_MAXV + 31) / 32) * 4 <= 2048, "penalty bitmap fits the histogram area");
static_assert(128 * sizeof(unsigned long long) <= 2048, "a warp list job's top-p search bins fit the histogram area");
// The CTA's list slab in global memory (lists of FLC..LCAP entries): indices,
// value keys, probabilities; F_SLAB_BYTES must fit one scratch stride.
constexpr size_t F_GL_VK = (size_t)LCAP * 2;
constexpr size_t F_GL_PV = F_GL_VK + (size_t)LCAP * 4;
constexpr size_t F_SLAB_BYTES = F_GL_PV + (size_t)LCAP * 8;
constexpr int F_MIN_SCRATCH_STRIDE = 16384;        // u64 per slab: >= F_SLAB_BYTES / 8 and >= a sort of LCAP keys
static_assert(F_SLAB_BYTES <= (size_t)F_MIN_SCRATCH_STRIDE * 8, "list slab fits a scratch stride");
static_assert(F_GL_PV % 8 == 0, "aligned slab probabilities");

// Dynamic shared memory of the fused kernel for rows of V logits: the fast
// path's buffers or the general path's layout, whichever is larger.
__host__ __device__ inline size_t fused_smem_bytes(int V) {
  const size_t g = layout_for(V).total;
  return g > F_FAST_BYTES ? g : F_FAST_BYTES;
}

// Phase trace (measurement builds only: -DC4S_TRACE): thread 0 of a CTA
// records clock64() at phase boundaries of its first rows.
#ifdef C4S_TRACE
constexpr int TR_CTAS = 1024, TR_ROWS = 16, TR_PH = 8;
__device__ long long g_trace[TR_CTAS * TR_ROWS * TR_PH];
__device__ int g_trace_info[TR_CTAS * TR_ROWS];
__device__ __forceinline__ void f_trace(int slot, int ph) {
  if (threadIdx.x == 0 && blockIdx.x < TR_CTAS && slot < TR_ROWS)
    g_trace[((int)blockIdx.x * TR_ROWS + slot) * TR_PH + ph] = clock64();
}
__device__ __forceinline__ void f_trace_info(int slot, int v) {
  if (threadIdx.x == 0 && blockIdx.x < TR_CTAS && slot < TR_ROWS) g_trace_info[(int)blockIdx.x * TR_ROWS + slot] = v;
}
#define C4S_TR(slot, ph) f_trace(slot, ph)
#define C4S_TR_INFO(slot, v) f_trace_info(slot, v)
#else
#define C4S_TR(slot, ph)
#define C4S_TR_INFO(slot, v)
#endif

struct FGeo {
  int V, shift, nq, seg;
};
__device__ __forceinline__ FGeo fgeo(int V, int shift) {
  FGeo g;
  g.V = V;
  g.shift = shift;
  const int nslot = (V + shift + 3) >> 2;
  g.seg = (((nslot + NWARP - 1) / NWARP) + 31) & ~31;
  g.nq = g.seg >> 5;
  return g;
}
__device__ __forceinline__ int fslot(const FGeo& g, int q) {
  return (threadIdx.x >> 5) * g.seg + 32 * q + (threadIdx.x & 31);
}
__device__ __forceinline__ float4 fload(const float* rb, int f) { return reinterpret_cast<const float4*>(rb)[f]; }

struct FShared {
  unsigned long long bar;
  MetaSlot meta[2];
  int nrow[2];
  unsigned redu[NWARP];
  int redi[NWARP];
  int abort_row;
  int lres;                                        // list job result (warp mode)
  int tslot;                                       // trace builds: the row's slot
  RowJob J;
  LRed R;
};

struct FList {
  unsigned short* li;
  unsigned* vk;
  double* pv;
  unsigned long long* hist;
  unsigned* bins;                                  // octave bins / staged positions (alias vk, pv)
};

// Candidates of a list held as element indices into the staged, penalised row.
struct RowKeys {
  const float* srow;
  const unsigned short* li;
  __device__ __forceinline__ unsigned val(int e) const { return fkey(srow[li[e]]); }
  __device__ __forceinline__ unsigned idx(int e) const { return li[e]; }
};

// Block sum of per-thread counts: every thread gets its warp's base and the
// total. S.redi is next written only behind later CTA barriers (the fill of
// the row's job record is followed by one), so no barrier closes this.
__device__ __forceinline__ int fblock_base(int cnt, FShared& S, int* total) {
  const int w = threadIdx.x >> 5;
  const int ws = __reduce_add_sync(FULL, cnt);
  if ((threadIdx.x & 31) == 0) S.redi[w] = ws;
  csync();
  int base = 0, t = 0;
#pragma unroll
  for (int k = 0; k < NWARP; ++k) {
    if (k < w) base += S.redi[k];
    t += S.redi[k];
  }
  *total = t;
  return base;
}

// Second pass for a warp whose candidates overflowed its staging: element
// indices selected by `sel`, in index order, from li[base]. Whole warp calls.
template <typename Sel>
__device__ __forceinline__ void f_write_list(unsigned short* li, int base, const float* rb, const FGeo& g, Sel sel) {
  int run = base;
  for (int q = 0; q < g.nq; ++q) {
    const int f = fslot(g, q);
    const float4 v = fload(rb, f);
    const int m = (sel(v.x) ? 1 : 0) | (sel(v.y) ? 2 : 0) | (sel(v.z) ? 4 : 0) | (sel(v.w) ? 8 : 0);
    if (__any_sync(FULL, m)) {
      int tot;
      int pos = run + warp_prefix4(__popc(m), &tot);
      const int i0 = 4 * f - g.shift;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (m & (1 << c)) li[pos++] = (unsigned short)(i0 + c);
      run += tot;
    }
  }
}

// One gather pass: each warp stages the buffer positions of the elements
// `sel` accepts, in index order, in its share of the bin area; once the warps'
// counts give their list offsets it copies them to li as element indices (a
// warp with more than F_STAGE_CAP writes its part with a second pass).
// With `track`, *xmx gets the largest element `sel` rejects (every thread).
// Lists of up to FLC entries go to shared memory (L.li), longer ones (up to
// LCAP) to the CTA's list slab in global memory (gli). Returns the list
// length (every thread), or -1 if it exceeds LCAP.
template <bool TRACK, typename Sel>
__device__ __forceinline__ int f_gather(const float* rb, const FGeo& g, FShared& S, FList L, unsigned short* gli,
                                        Sel sel, float* xmx) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned short* stage = reinterpret_cast<unsigned short*>(L.bins + warp * F_WSTRIDE);
  int run = 0;
  float mx = -INFINITY;
#pragma unroll 3
  for (int q = 0; q < g.nq; ++q) {
    const int f = fslot(g, q);
    const float4 v = fload(rb, f);
    int m = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float x = f4c(v, c);
      if (sel(x)) m |= 1 << c;
      else if (TRACK) mx = fmaxf(mx, x);
    }
    if (__any_sync(FULL, m)) {
      int tot;
      int pos = run + warp_prefix4(__popc(m), &tot);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (m & (1 << c)) {
          if (pos < F_STAGE_CAP) stage[pos] = (unsigned short)(4 * f + c);
          ++pos;
        }
      }
      run += tot;
    }
  }
  if (TRACK) {
    const unsigned km = __reduce_max_sync(FULL, fkey(mx));
    if (lane == 0) S.redu[warp] = km;
  }
  int ng;
  const int base = fblock_base(lane == 0 ? run : 0, S, &ng);   // its barriers also publish S.redu
  if (TRACK) {
    unsigned kx = S.redu[0];
#pragma unroll
    for (int w = 1; w < NWARP; ++w) kx = kx > S.redu[w] ? kx : S.redu[w];
    *xmx = fkey_inv(kx);
  }
  if (ng > LCAP) return -1;
  unsigned short* li = ng <= FLC ? L.li : gli;
  if (run <= F_STAGE_CAP) {
    __syncwarp();
    for (int i = lane; i < run; i += 32) li[base + i] = (unsigned short)(stage[i] - g.shift);
  } else {
    f_write_list(li, base, rb, g, sel);
  }
  return ng;
}

// The smallest x with oct(x) <= bl (it exists: oct(m_x) = 0), by a 32-way
// search over the float order between -inf (octave NOCT > bl) and m_x: each
// step every lane probes one point, and the ballot narrows the range 33-fold.
// The predicate is monotone in x (see oct_of_t). Whole warp calls.
__device__ __forceinline__ float list_threshold_w(const RowCtx& rc, int bl) {
  const int lane = threadIdx.x & 31;
  unsigned lo = fkey(-INFINITY), hi = fkey(rc.m_x);      // pred(lo) false, pred(hi) true
  while (hi - lo > 1u) {
    const unsigned span = hi - lo;
    const unsigned mid = lo + (unsigned)(((unsigned long long)span * (unsigned)(lane + 1)) / 33ull);
    const bool p = mid != lo && oct_of_t(oct_t(rc, fkey_inv(mid))) <= bl;
    const unsigned b = __ballot_sync(FULL, p);
    if (b == 0u) {
      lo = __shfl_sync(FULL, mid, 31);
    } else {
      const int L = __ffs(b) - 1;
      const unsigned nh = __shfl_sync(FULL, mid, L);
      const unsigned nl = __shfl_sync(FULL, mid, L > 0 ? L - 1 : 0);
      hi = nh;
      if (L > 0) lo = nl > lo ? nl : lo;
    }
  }
  return fkey_inv(hi);
}

// Top-k row: the list of elements >= the maxima threshold (at least k of
// them, every one that can survive top-k). Returns its length, or -1.
__device__ __forceinline__ int f_topk_list_body(const RowCtx& rc, const float* rb, const FGeo& g, FShared& S,
                                                const FList& L, unsigned short* gli, int k, bool two, float tm,
                                                float t2) {
  // a warp whose kw-th largest lane maximum (of the two largest per lane when
  // `two`) is finite has >= kw elements >= it, so >= k elements are >= tau,
  // the smallest over the warps (-inf: not enough elements; general path)
  if (k > NT * (two ? 2 : 1)) return -1;
  const float tau = u_threshold<NT>(tm, t2, two, rc.m_x, k, L.bins, &S.redu[0], [] { csync(); }, true);
  // fl(x/T) merges x only with values at most |x| 2^-23 below it: lowering tau
  // by 2^-18 relative (+ 2^-18 absolute) keeps every x tied with tau after /T
  const float tau_lo = tau - (fabsf(tau) + 1.0f) * 3.814697265625e-06f;
  if (!(tau_lo > -INFINITY)) return -1;
  float unused;
  return f_gather<false>(rb, g, S, L, gli, [&](float x) { return x >= tau_lo; }, &unused);
}
__device__ __noinline__ int f_topk_list(const RowCtx rc, const float* rb, const FGeo g, FShared& S, FList L,
                                        unsigned short* gli, int k, bool two, float tm, float t2) {
  return f_topk_list_body(rc, rb, g, S, L, gli, k, two, tm, t2);
}

// Row without top-k (top-p over the whole row, sampling.cpp:42-71): octave
// histogram of the estimates, the list down to the crossing octave (deeper
// while it stays short), the estimated tail and its bound into S.J. Returns
// the list length, or -1 (general path).
__device__ __noinline__ int f_k0_list(const Args& a, const RowCtx rc, const float* rb, const FGeo g, FShared& S,
                                      FList L, unsigned short* gli) {
  const int V = a.V;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (!(rc.thr > 0.0) || (a.debug & C4S_DEBUG_FORCE_BINS)) return -1;   // top_p >= 1, forced binned path
  unsigned* wb = L.bins + warp * F_WSTRIDE;
#pragma unroll
  for (int r = 0; r < FHREP; ++r) wb[r * 33 + lane] = 0u;
  __syncwarp();
  unsigned* hrep = wb + (lane & (FHREP - 1)) * 33;   // fewer lanes per bin address
#pragma unroll 3
  for (int q = 0; q < g.nq; ++q) {
    const float4 v = fload(rb, fslot(g, q));
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      // octave b = oct_of_t(t) and the estimate's mass in units of 2^-(b+20),
      // truncated: 2^(b - ns) 2^20 with ns = RN(-t log2 e); b - ns is exact
      // (in (-1, 0] below NOCT), so the error is ex2.approx's own plus the
      // rounding of ns, inside the 2 + 1.16 |t| ulp that the estimate's bound
      // allows for an exponential of t, and truncation loses below 2^-19 of
      // an element below NOCT. Below 2^21 per element, a replica's u32 bin
      // (at most 2^10 elements) cannot overflow; padding (-inf) gives 0.
      const float ns = oct_t(rc, f4c(v, c)) * -1.4426950408889634f;
      const int b = (int)fminf(ns, (float)NOCT);
      const unsigned m = (unsigned)(ex2_approx((float)b - ns) * 1048576.0f);
      if (m) atomicAdd(&hrep[b], m);
    }
  }
  csync();
  // every warp: lane b holds octave b's mass; suffix sums give the mass below
  // each octave, ballots the crossing octave and the list's last octave
  double o = 0.0;
  if (lane <= NOCT) {
    unsigned long long qs = 0ull;
#pragma unroll
    for (int w = 0; w < NWARP; ++w)
#pragma unroll
      for (int r = 0; r < FHREP; ++r) qs += L.bins[w * F_WSTRIDE + r * 33 + lane];
    o = ldexp((double)qs, -(lane + 20));
  }
  const double wo = o * oct_d(lane <= NOCT ? lane : NOCT);
  double suf = o, wsuf = wo;                        // sums over octaves >= lane
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const double t1 = __shfl_down_sync(FULL, suf, off), t2d = __shfl_down_sync(FULL, wsuf, off);
    if (lane + off < 32) { suf += t1; wsuf += t2d; }
  }
  double pre = o * ldexp(1.0, lane + 1);            // count bound of octaves <= lane
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const double t = __shfl_up_sync(FULL, pre, off);
    if (lane >= off) pre += t;
  }
  const double Se = __shfl_sync(FULL, suf, 0);
  const double below = __shfl_down_sync(FULL, suf, 1), wbelow = __shfl_down_sync(FULL, wsuf, 1);
  const double blw = lane < 31 ? below : 0.0, wblw = lane < 31 ? wbelow : 0.0;   // octaves > lane
  const double Th = rc.thr * Se;
  const double rnd = 2.0 * ((4.0 * V + 16.0) * U53 * Se);
  const double es = est_err(Se, __shfl_sync(FULL, wsuf, 0), rc.m_y, 33, V);
  int bl = -1;
  {
    // crossing octave: suffix sum (from the deep end) first exceeds Th
    const unsigned cr = __ballot_sync(FULL, lane <= NOCT && suf > Th);
    const int bc = cr ? 31 - __clz(cr) : -1;
    if (bc < 0 || bc == NOCT) {
      csync();                                     // every warp has read the bins
      return -1;
    }
    // the list: octaves 0..bl, bl >= bc the first whose tail is clearly below Th
    const bool okl = lane >= bc && lane < NOCT && blw + 2.0 * est_err(blw, wblw, rc.m_y, 33, V) + rc.thr * es + rnd < Th;
    const unsigned lb = __ballot_sync(FULL, okl);
    bl = lb ? __ffs(lb) - 1 : -1;
    if (bl >= 0) {
      // go deeper while the list stays short, until the tail is below Th/64:
      // the list job's decision band (which scales with the tail) then
      // rarely reaches the crossing element
      const unsigned small = __ballot_sync(FULL, lane >= bl && lane < NOCT && blw <= Th * 0.015625);
      const unsigned fits = __ballot_sync(FULL, lane >= bl && lane < NOCT && pre <= 0.5 * LIST_DEEP);
      const int bt = small ? __ffs(small) - 1 : NOCT - 1;
      const int bf = fits ? 31 - __clz(fits) : bl;
      bl = max(bl, min(bt, bf));
    }
  }
  const double nb = bl >= 0 ? __shfl_sync(FULL, pre, bl) : 0.0;
  const double tl = bl >= 0 ? __shfl_sync(FULL, blw, bl) : 0.0;
  const double tl_err = bl >= 0 ? est_err(tl, __shfl_sync(FULL, wblw, bl), rc.m_y, 33, V) : 0.0;
  // the list: elements in octaves <= bl, i.e. >= x*, in index order
  const float xs = bl >= 0 ? list_threshold_w(rc, bl) : 0.0f;
  csync();                                         // every warp has read the bins: they become staging
  if (bl < 0 || nb > 2.0 * LCAP) return -1;
  float xm;
  const int ng = f_gather<true>(rb, g, S, L, gli, [&](float x) { return x >= xs; }, &xm);
  if (threadIdx.x == 0) {
    S.J.tail = tl;
    S.J.tail_err = tl_err;
    S.J.ykex = xm > -INFINITY ? fkey(yex(rc, xm)) : 0u;
  }
  return ng;
}

// Exact tail of a row without top-k, from the staged penalised row: the sum
// of exp((double)(y - m_y)) over every element below the list (each tempered
// as the reference does, re-associated: its rounding is inside the list's
// double-sum band; each term by exp_tail, within 2^-51 of the reference's, so
// tail_err = 2^-50 tail), in place of the estimate.
__device__ __noinline__ void f_exact_tail(const Args& a, const float* rb, const FGeo g, FShared& S) {
  const float T = S.J.T;
  const bool do_t = T != 1.0f;
  const float rT = do_t ? __frcp_rn(T) : 1.0f;
  const unsigned ykex = S.J.ykex;
  const float m_y = S.J.m_y;
  double t[4] = {0.0, 0.0, 0.0, 0.0};               // one sum per float4 lane: four exp_tail chains in flight
  unsigned long long redo = 0ull;                   // elements whose quotient div_rn_try could not prove
  auto term = [&](float x, float y) {
    return (x > -INFINITY && fkey(y) <= ykex) ? exp_tail(__fsub_rn(y, m_y), S.R.tab) : 0.0;
  };
  for (int q = 0; q < g.nq; ++q) {
    const float4 v = fload(rb, fslot(g, q));
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float x = f4c(v, c);
      bool ok = true;
      const float y = (do_t && x > -INFINITY) ? div_rn_try(x, T, rT, ok) : x;
      if (ok) t[c] += term(x, y);
      else redo |= 1ull << (4 * q + c);
    }
  }
  for (; redo; redo &= redo - 1ull) {
    const int b = __ffsll(redo) - 1;
    const float x = f4c(fload(rb, fslot(g, b >> 2)), b & 3);
    t[0] += term(x, div_call(x, T));
  }
  const double tail = LG<true>::sum((t[0] + t[1]) + (t[2] + t[3]), S.R);
  if (threadIdx.x == 0) {
    S.J.tail = tail;
    S.J.tail_err = ldexp(tail, -50);
    atomicAdd(&a.counters[C4S_CNT_EXACT_TAIL], 1ull);
  }
  csync();
}

// Ascending order of the warp's 64 distinct keys (lane l holds positions 2l
// and 2l+1): each key's rank is the number of smaller keys, counted over
// all 64 by shuffles (32 independent steps, no compare-exchange chain), and
// the keys are scattered to their ranks in `buf` (64 u64 of shared memory)
// and read back in order. Whole warp calls.
__device__ __forceinline__ void warp_rank_sort2(unsigned long long (&k)[2], unsigned long long* buf) {
  const int lane = threadIdx.x & 31;
  int r0 = 0, r1 = 0;
#pragma unroll 8
  for (int s = 0; s < 32; ++s) {
    const unsigned long long o0 = __shfl_sync(FULL, k[0], s), o1 = __shfl_sync(FULL, k[1], s);
    r0 += (o0 < k[0] ? 1 : 0) + (o1 < k[0] ? 1 : 0);
    r1 += (o0 < k[1] ? 1 : 0) + (o1 < k[1] ? 1 : 0);
  }
  buf[r0] = k[0];
  buf[r1] = k[1];
  __syncwarp();
  k[0] = buf[2 * lane];
  k[1] = buf[2 * lane + 1];
  __syncwarp();
}

// The list job of a list of at most 64 entries, by one warp with the list in
// registers (lane l holds list positions 2l and 2l+1; positions are in index
// order): tempered value keys; one ascending register sort of (value key,
// position) gives the k-th largest value (top-k, sampling.cpp:30-40) and the
// canonical top-p order (sampling.cpp:42-71); exact double probabilities of
// the survivors; the top-p crossing on a prefix scan from the tail mass; the
// draw (text2semantic.cpp:150-165) on a prefix scan in index order. Every
// decision is the one list_job takes; when one of them falls inside its
// rounding band (or the debug flags force the slow paths) it returns false
// without writing anything, and the caller runs list_job instead. `tab` is
// exp_tail's table in shared memory; pvs holds at least 128 doubles (the
// sort's scatter buffer follows the 64 probabilities).
__device__ __forceinline__ bool f_short_job_body(const Args& a, int row, RowJob& J, const float* srow,
                                                 const unsigned short* li, double* pvs, const double* tab) {
  const int lane = threadIdx.x & 31;
  const int n = J.n, k = J.k;
  const bool k0 = J.kind == JOB_K0;
  if (n > 64 || (a.debug & (C4S_DEBUG_FORCE_BINS | C4S_DEBUG_FORCE_REFINE))) return false;
  const float T = J.T;
  const bool do_t = T != 1.0f;
  const float rT = do_t ? __frcp_rn(T) : 1.0f;
  const float m_y = J.m_y;
  unsigned vkey[2], idx[2];
  unsigned lmin = ~0u, lmax = 0u;
  float xs[2];
  bool ok[2] = {true, true};
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int p = 2 * lane + j;
    vkey[j] = 0u;
    idx[j] = 0u;
    xs[j] = 0.0f;
    if (p < n) {
      idx[j] = li[p];
      xs[j] = srow[idx[j]];
      vkey[j] = fkey(do_t ? div_rn_try(xs[j], T, rT, ok[j]) : xs[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    if (!ok[j]) vkey[j] = fkey(div_call(xs[j], T));  // rare: the quotient div_rn_try could not prove
    if (2 * lane + j < n) {
      lmin = min(lmin, vkey[j]);
      lmax = max(lmax, vkey[j]);
    }
  }
  const unsigned vmin = __reduce_min_sync(FULL, lmin), vmax = __reduce_max_sync(FULL, lmax);
  if (k0 && J.ykex >= vmin) return false;         // list_job hands such a row to the general path
  // ascending (value key, position); padding (key = its position, below
  // every element's key: value keys are >= 1) sorts first
  unsigned long long sk[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const unsigned p = 2 * lane + j;
    sk[j] = (int)p < n ? ((unsigned long long)vkey[j] << 32) | p : (unsigned long long)p;
  }
  warp_rank_sort2(sk, reinterpret_cast<unsigned long long*>(pvs + 64));
  auto at = [&](int pos) {                          // sorted key at position pos (uniform)
    return __shfl_sync(FULL, (pos & 1) ? sk[1] : sk[0], pos >> 1);
  };
  unsigned tk = vmin;
  if (k > 0 && k < n && vmin != vmax) tk = (unsigned)(at(64 - k) >> 32);
  // probabilities of the survivors, in sorted order (Tang's exp_tail, within
  // 2^-51 of the reference's exp: every decision below is checked against a
  // band that covers it), also stored by list position for the draw
  double pr[2];
  int nl = 0;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const unsigned v = (unsigned)(sk[j] >> 32);
    const bool real = v != 0u;                      // not padding
    const bool sv = real && v >= tk;
    pr[j] = sv ? exp_tail(__fsub_rn(fkey_inv(v), m_y), tab) : 0.0;
    if (real) pvs[(int)(sk[j] & 0xffffffffull)] = pr[j];
    nl += sv ? 1 : 0;
  }
  const double ps = warp_sum_d(pr[0] + pr[1]);
  const int ns = __reduce_add_sync(FULL, nl);
  const unsigned long long s63 = at(63);             // the largest survivor: (vmax, last position)
  const unsigned long long kmax = (s63 & 0xffffffff00000000ull) | li[(int)(s63 & 0xffffffffull)];
  const double thr = J.thr, St = J.tail + ps;
  unsigned long long kst;
  if (thr < 0.0) {
    kst = 0ull;                                     // p > 1: nothing removed
  } else if (thr == 0.0) {
    // p == 1: only zero probabilities go, which exp_tail (0 below -700) does
    // not tell apart from the reference's smallest ones: list_job decides
    return false;
  } else {
    // the first sorted position whose running mass from the tail exceeds Th
    const double Th = thr * St;
    const double ls = pr[0] + pr[1];
    double incl = ls;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(FULL, incl, o);
      if (lane >= o) incl += y;
    }
    double run = J.tail + incl - ls, bf = 0.0, cu = 0.0;
    int hj = -1;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const double nx = run + pr[j];
      if (hj < 0 && pr[j] > 0.0 && nx > Th) { hj = j; bf = run; cu = nx; }
      run = nx;
    }
    const unsigned cb = __ballot_sync(FULL, hj >= 0);
    if (!cb) return false;                          // no crossing: list_job's exact path
    const int L = __ffs(cb) - 1;
    const int jL = __shfl_sync(FULL, hj, L);
    const double before = __shfl_sync(FULL, bf, L), cur = __shfl_sync(FULL, cu, L);
    const unsigned long long ck = at(2 * L + jL);
    const double bd = 2.0 * ((4.0 * (k0 ? a.V : ns) + 16.0) * U53 * St) + 2.0 * J.tail_err;
    if (!(before <= Th - bd && cur > Th + bd)) return false;
    kst = (ck & 0xffffffff00000000ull) | li[(int)(ck & 0xffffffffull)];
  }
  kst = kst < kmax ? kst : kmax;                    // min_tokens_to_keep = 1
  // the draw, in index order (list positions)
  int tok = 0;
  if (J.u53 != 0ull) {
    __syncwarp();                                   // pvs written in sorted order, read by position
    double q[2];
    int kl = 0;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const unsigned long long yk = ((unsigned long long)vkey[j] << 32) | idx[j];
      const bool kept = 2 * lane + j < n && vkey[j] >= tk && yk >= kst;
      q[j] = kept ? pvs[2 * lane + j] : 0.0;
      kl += kept ? 1 : 0;
    }
    const double ls = q[0] + q[1];
    double incl = ls;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(FULL, incl, o);
      if (lane >= o) incl += y;
    }
    const double s2 = __shfl_sync(FULL, incl, 31);
    const int nk = __reduce_add_sync(FULL, kl);
    const double r = J.u * s2;
    double acc = incl - ls, pv0 = 0.0, cv0 = 0.0;
    int fj = -1;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const double nx = acc + q[j];
      if (fj < 0 && q[j] > 0.0 && nx >= r) { fj = j; pv0 = acc; cv0 = nx; }
      acc = nx;
    }
    const unsigned fb = __ballot_sync(FULL, fj >= 0);
    if (!fb) return false;
    const int L = __ffs(fb) - 1;
    const int jL = __shfl_sync(FULL, fj, L);
    const double prev = __shfl_sync(FULL, pv0, L), cur = __shfl_sync(FULL, cv0, L);
    const double bd2 = 2.0 * ((4.0 * nk + 16.0) * U53 * s2);
    if (!(prev < r - bd2 && cur > r + bd2)) return false;
    tok = (int)__shfl_sync(FULL, jL ? idx[1] : idx[0], L);
  }
  if (lane == 0) {
    a.out_ids[row] = tok;
    a.rng[row] = J.xs;
    J.kstar = kst;
    J.thresh_key = k > 0 ? tk : 0u;
    J.status = RES_DONE;
  }
  __syncwarp();
  return true;
}

__device__ __noinline__ bool f_short_job(const Args& a, int row, RowJob& J, const float* srow,
                                         const unsigned short* li, double* pvs, const double* tab) {
  return f_short_job_body(a, row, J, srow, li, pvs, tab);
}

// list_job on a list of at most 256 entries, by one warp (out of line).
__device__ __noinline__ bool f_warp_list_job(const Args& a, int row, const float* srow, FShared& S, FList L,
                                             unsigned long long* sb, bool refine) {
  return list_job<false, true, RowKeys>(a, row, S.J, RowKeys{srow, L.li}, sb, L.vk, L.pv, L.hist, refine, S.R,
                                        nullptr);
}

// The list job on a short list, by warp 0 (the other warps wait at the
// barrier). INL: the register-resident short job inlined into the caller
// (the small-batch kernel, which has the registers for it).
template <bool INL>
__device__ __forceinline__ void f_list_warp_body(const Args& a, int row, const float* srow, FShared& S,
                                                 const FList& L, unsigned long long* sb, bool refine) {
  if ((threadIdx.x >> 5) == 0) {
    bool ok = false;
    if (!refine) {
      if constexpr (INL) ok = f_short_job_body(a, row, S.J, srow, L.li, L.pv, S.R.tab);
      else ok = f_short_job(a, row, S.J, srow, L.li, L.pv, S.R.tab);
    }
    if (!ok) ok = f_warp_list_job(a, row, srow, S, L, sb, refine);
    if (threadIdx.x == 0) S.lres = ok ? 1 : 0;
  }
  csync();
}
__device__ __noinline__ void f_list_warp(const Args& a, int row, const float* srow, FShared& S, FList L,
                                         unsigned long long* sb, bool refine) {
  f_list_warp_body<false>(a, row, srow, S, L, sb, refine);
}

// The list job on a long list, by the whole CTA; li/vk/pv in shared memory
// (up to FLC entries) or in the CTA's list slab in global memory.
__device__ __noinline__ void f_list_cta(const Args& a, int row, const float* srow, FShared& S,
                                        const unsigned short* li, unsigned* vk, double* pv, unsigned long long* hist,
                                        unsigned long long* sb, bool refine) {
  const bool ok = list_job<true, true, RowKeys>(a, row, S.J, RowKeys{srow, li}, sb, vk, pv, hist, refine, S.R,
                                                nullptr);
  if (threadIdx.x == 0) S.lres = ok ? 1 : 0;
  csync();
}

// Processed logits of a finished list row: tempered values, with what top-k
// (threshold key tk) and top-p (keys below kst) removed set to -inf.
__device__ __noinline__ void f_write_masked(const Args& a, int row, const float* rb, const FGeo g, const RowCtx rc,
                                            unsigned tk, unsigned long long kst) {
  float* o = a.out_logits + (long long)row * a.out_ld;
  for (int q = 0; q < g.nq; ++q) {
    const int f = fslot(g, q);
    const float4 v = fload(rb, f);
    const int i0 = 4 * f - g.shift;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int i = i0 + c;
      if ((unsigned)i < (unsigned)g.V) {
        const float y = yex(rc, f4c(v, c));
        o[i] = (fkey(y) < tk || (y > -INFINITY && ckey(y, i) < kst)) ? -INFINITY : y;
      }
    }
  }
}

// The raw (penalised) row, for greedy rows' processed logits.
__device__ __noinline__ void f_write_raw(const Args& a, int row, const float* rb, const FGeo g) {
  float* o = a.out_logits + (long long)row * a.out_ld;
  for (int q = 0; q < g.nq; ++q) {
    const int f = fslot(g, q);
    const float4 v = fload(rb, f);
    const int i0 = 4 * f - g.shift;
#pragma unroll
    for (int c = 0; c < 4; ++c)
      if ((unsigned)(i0 + c) < (unsigned)g.V) o[i0 + c] = f4c(v, c);
  }
}

enum { F_DONE = 0, F_GENERAL = 1 };

// One staged, penalised row on the fast path. Returns F_DONE (id, state and
// processed logits written) or F_GENERAL.
template <bool INL>
__device__ __forceinline__ int f_row_body(const Args& a, int row, const MetaSlot& M, const float* rb, const FGeo& g,
                                          FShared& S, const FList& L) {
  const int V = a.V;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const c4s_row_params P = M.P;
  const int k = P.top_k;
  const bool do_k = k > 0 && k < V;
  const bool two = !P.greedy && do_k && k > NWARP * 32 / 2;   // the two largest per lane seed the list

  // ---- row max, per-lane maxima (and second maxima) ----
  // (top-k rows: the threshold histogram's bins are cleared here, ordered
  // before their use by the barrier of the max reduction)
  if (!P.greedy && do_k) L.bins[tid] = 0u;
  static_assert(NT == 256, "one bin per thread");
  float tm = -INFINITY, t2 = -INFINITY;
#pragma unroll 3
  for (int q = 0; q < g.nq; ++q) {
    const float4 v = fload(rb, fslot(g, q));
    if (two) {
      t2 = fmaxf(t2, fminf(tm, v.x)); tm = fmaxf(tm, v.x);
      t2 = fmaxf(t2, fminf(tm, v.y)); tm = fmaxf(tm, v.y);
      t2 = fmaxf(t2, fminf(tm, v.z)); tm = fmaxf(tm, v.z);
      t2 = fmaxf(t2, fminf(tm, v.w)); tm = fmaxf(tm, v.w);
    } else {
      tm = fmaxf(tm, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
    }
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
  C4S_TR(S.tslot, 3);

  RowCtx rc;
  rc.row = row; rc.V = V; rc.i0 = 0;
  rc.T = P.temperature;
  rc.do_t = !(rc.T == 1.0f || rc.T <= 0.0f);

  // ---- greedy: first index of the max (sampling.cpp:73-76) ----
  if (P.greedy) {
    csync();                                       // every warp has read S.redu
    unsigned cand = 0xffffffffu;
    if (m_x > -INFINITY && tm == m_x) {
      for (int q = 0; q < g.nq; ++q) {
        const int f = fslot(g, q);
        const float4 v = fload(rb, f);
        const int i0 = 4 * f - g.shift;
        if (v.w == m_x) cand = min(cand, (unsigned)(i0 + 3));
        if (v.z == m_x) cand = min(cand, (unsigned)(i0 + 2));
        if (v.y == m_x) cand = min(cand, (unsigned)(i0 + 1));
        if (v.x == m_x) cand = min(cand, (unsigned)i0);
        if (cand != 0xffffffffu) break;              // later slots hold larger indices
      }
    }
    cand = __reduce_min_sync(FULL, cand);
    if (lane == 0) S.redu[warp] = cand;
    csync();
    if (tid == 0) {
      unsigned b = S.redu[0];
      for (int w = 1; w < NWARP; ++w) b = S.redu[w] < b ? S.redu[w] : b;
      a.out_ids[row] = b == 0xffffffffu ? 0 : (int)b;
    }
    if (a.out_logits) f_write_raw(a, row, rb, g);
    csync();
    return F_DONE;
  }

  // ---- sampled rows: preconditions ----
  if (!(m_x > -INFINITY && m_x < INFINITY)) return F_GENERAL;
  rc.m_x = m_x;
  rc.m_y = rc.do_t ? __fdiv_rn(m_x, rc.T) : m_x;
  rc.rT = rc.do_t ? __frcp_rn(rc.T) : 1.0f;
  if (!(fabsf(rc.m_y) < 262144.0f)) return F_GENERAL;
  if (P.min_tokens_to_keep != 1) return F_GENERAL;
  if (a.debug & C4S_DEBUG_FORCE_EXACT) return F_GENERAL;
  rc.thr = __dsub_rn(1.0, (double)P.top_p);
  {
    unsigned long long xs = M.rng;
    xs ^= xs << 13; xs ^= xs >> 7; xs ^= xs << 17;
    rc.xs = xs;
    rc.u53 = xs >> 11;
    rc.u = (double)rc.u53 * 1.1102230246251565e-16;   // (x>>11) / 2^53, exact
  }

  // ---- the candidate list ----
  // the CTA's two scratch slabs: the exact fallback's sort buffer, then the
  // list slab of lists longer than FLC (element indices, value keys, probabilities)
  unsigned long long* sb = a.scratch + (size_t)blockIdx.x * (size_t)a.scratch_stride;
  unsigned char* slab = reinterpret_cast<unsigned char*>(a.scratch + (size_t)(gridDim.x + blockIdx.x) * (size_t)a.scratch_stride);
  unsigned short* gli = reinterpret_cast<unsigned short*>(slab);
  unsigned* gvk = reinterpret_cast<unsigned*>(slab + F_GL_VK);
  double* gpv = reinterpret_cast<double*>(slab + F_GL_PV);
  int ng;
  if constexpr (INL) ng = do_k ? f_topk_list_body(rc, rb, g, S, L, gli, k, two, tm, t2) : f_k0_list(a, rc, rb, g, S, L, gli);
  else ng = do_k ? f_topk_list(rc, rb, g, S, L, gli, k, two, tm, t2) : f_k0_list(a, rc, rb, g, S, L, gli);
  if (ng < 0) return F_GENERAL;
  if (tid == 0) {
    fill_job(S.J, rc, do_k ? JOB_TOPK : JOB_K0, ng, do_k ? k : 0);
    if (do_k) {
      S.J.tail = 0.0;
      S.J.tail_err = 0.0;
      S.J.ykex = 0u;
    }
  }
  csync();
  C4S_TR(S.tslot, 4);
  C4S_TR_INFO(S.tslot, (ng << 4) | (do_k ? 1 : 2));

  // ---- the list job in place, an exact tail if its band needs one ----
  const float* srow = rb + g.shift;
  for (int pass = 0; pass < 2; ++pass) {
    const bool refine = pass == 1;
    if (ng <= 256) {
      if constexpr (INL) f_list_warp_body<true>(a, row, srow, S, L, sb, refine);
      else f_list_warp(a, row, srow, S, L, sb, refine);
    }
    else if (ng <= FLC) f_list_cta(a, row, srow, S, L.li, L.vk, L.pv, L.hist, sb, refine);
    else f_list_cta(a, row, srow, S, gli, gvk, gpv, L.hist, sb, refine);
    C4S_TR(S.tslot, 5 + pass);
    if (S.lres) break;
    if (refine || S.J.status != RES_REFINE) return F_GENERAL;
    f_exact_tail(a, rb, g, S);
  }
  if (a.out_logits) f_write_masked(a, row, rb, g, rc, S.J.thresh_key, S.J.kstar);
  csync();
  return F_DONE;
}
__device__ __noinline__ int f_row(const Args& a, int row, const MetaSlot& M, const float* rb, const FGeo g,
                                  FShared& S, FList L) {
  return f_row_body<false>(a, row, M, rb, g, S, L);
}

// Fused persistent kernel: rows handed out dynamically (the first G
// statically), each finished in its CTA. Three forms: MINB = 3 resident CTAs
// per SM with the per-row paths out of line (batches above two rows per SM);
// MINB = 1, one CTA per SM with every register it needs and the common path
// (top-k row, short list) inlined: no spills and no call frames on the
// latency-bound path of small batches (B <= SMs, B = 1 among them); and
// MINB = 2 with the same inlining for batches of up to two rows per SM.
template <int MINB, bool INL>
__global__ void __launch_bounds__(NT, MINB) fused_kernel_t(Args a) {
  extern __shared__ __align__(128) unsigned char fsm[];
  __shared__ FShared S;
  __shared__ Shared GS;                             // general path
  __shared__ Args sa;                               // the out-of-line paths read the arguments from here
  float* rb = reinterpret_cast<float*>(fsm);
  FList L;
  L.li = reinterpret_cast<unsigned short*>(fsm + FL_LI);
  L.vk = reinterpret_cast<unsigned*>(fsm + FL_VK);
  L.pv = reinterpret_cast<double*>(fsm + FL_PV);
  L.hist = reinterpret_cast<unsigned long long*>(fsm + FL_HIST);
  L.bins = reinterpret_cast<unsigned*>(fsm + FL_VK);
  const Layout GL = layout_for(a.V);
  const int V = a.V;
  const int tid = threadIdx.x;
  const int G = gridDim.x;
  unsigned* ctr = a.defer_cnt;                     // [0] row tickets, [1] CTAs done

  if (tid < 64) S.R.tab[tid] = EXP2_J64[tid];
  if (tid == 0) {
    mbar_init(&S.bar, 1);
    mbar_init(&GS.bar, 1);
    sa = a;
  }
  auto fill_ninf = [&]() {
    const float4 ninf = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    for (int i = tid; i < F_SLOTS; i += NT) reinterpret_cast<float4*>(rb)[i] = ninf;
  };
  fill_ninf();
  int act_pend = 1;
  auto issue_meta = [&](int r, MetaSlot& ms) {
    if (r >= a.B) return;
    const char* prm = reinterpret_cast<const char*>(a.params + (long long)r * a.params_stride);
    if (tid < 3) cp_async8(reinterpret_cast<char*>(&ms.P) + 8 * tid, prm + 8 * tid);
    else if (tid == 3) { if (a.hist_off) cp_async8(&ms.off0, a.hist_off + r); else ms.off0 = 0; }
    else if (tid == 4) {
      if (a.hist_len) cp_async4(&ms.hlen, a.hist_len + r);
      else if (a.hist_off) cp_async8(&ms.off1, a.hist_off + r + 1);
      else ms.off1 = 0;
    }
    else if (tid == 5) cp_async8(&ms.rng, a.rng + r);
    else if (tid == 6) act_pend = a.active ? (int)a.active[r] : 1;
  };
  // one CTA takes the rows in order; several take tickets (the first row statically)
  const bool tickets = G > 1;
  csync();                                         // the buffer is filled before the first copy lands
  // the previous kernel of the stream may write the logits (a head GEMM), the
  // RNG states and the counters: wait for it, then issue the first row's copy
  // at once, in parallel with its metadata
  grid_dep_wait();
  grid_dep_launch();
  const int r0 = blockIdx.x;
  Staged sg = stage_row(a.logits + (long long)r0 * a.ld, V, rb, &S.bar);
  if (tid == 0) S.nrow[0] = tickets ? G + (int)atomicAdd(&ctr[0], 1u) : r0 + 1;
  issue_meta(r0, S.meta[0]);
  cp_async_commit();
  if (tid == 6 && r0 < a.B) S.meta[0].active = act_pend;
  cp_async_wait<0>();
  csync();
  unsigned phase = 0, gphase = 0;

  int j = 0;
  int lost0 = a.B, lost1 = a.B;                    // rows this CTA holds when a bounded wait gave up
  for (int row = r0; row < a.B; ++j) {
    C4S_TR(j, 0);
    if (tid == 0) S.tslot = j;
    const MetaSlot& cur = S.meta[j & 1];
    MetaSlot& nxt = S.meta[(j + 1) & 1];
    const int next = S.nrow[j & 1];
    issue_meta(next, nxt);
    cp_async_commit();
    if (tid == 32 && next < a.B) prefetch_row(a.logits + (long long)next * a.ld, V);
    if (tid == 6 && next < a.B) nxt.active = act_pend;
    if (!cur.active && sg.body > 0) {
      // an inactive first row was staged before its metadata arrived: let the
      // copy complete (bounded) so that the barrier's phase stays in step
      if (tid == 0) {
        S.abort_row = mbar_wait_bounded(&S.bar, phase) ? 0 : 1;
        if (S.abort_row) atomicOr(a.errflags, C4S_DEVERR_TIMEOUT);
      }
      phase ^= 1u;
      csync();
      if (S.abort_row) {
        if (tid == 0) mbar_wait_bounded(&S.bar, phase ^ 1u);
        lost0 = row;
        lost1 = next;
        break;
      }
    }
    if (cur.active) {
      const c4s_row_params P = cur.P;
      const bool pen = a.hist_off && P.repetition_penalty != 1.0f;
      long long h0 = 0, h1 = 0;
      if (pen) {
        h0 = cur.off0;
        h1 = a.hist_len ? h0 + cur.hlen : cur.off1;
        if (h0 < 0 || h1 < h0 || h1 > a.hist_total) {
          if (tid == 0) atomicOr(a.errflags, C4S_DEVERR_HIST_RANGE);
          h0 = h1 = 0;
        }
      }
      const bool longh = h1 - h0 > F_HIST_WORDS;   // beyond the ids held in registers: bitmap
      unsigned* bm = reinterpret_cast<unsigned*>(L.hist);
      if (longh)
        for (int w = tid; w < (V + 31) / 32; w += NT) bm[w] = 0u;
      // the first 8 ids per thread in flight while the row arrives
      int hid[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const long long jj = h0 + tid + (long long)q * NT;
        hid[q] = jj < h1 ? a.hist[jj] : -1;
      }
      if (tid == 0) {
        bool ok = true;
        if (sg.body > 0) ok = mbar_wait_bounded(&S.bar, phase);
        S.abort_row = ok ? 0 : 1;
        if (!ok) atomicOr(a.errflags, C4S_DEVERR_TIMEOUT);
      }
      if (sg.body > 0) phase ^= 1u;
      if (sg.hpos >= 0) rb[sg.hpos] = sg.hval;
      // positions the previous row's shift filled but this row's does not
      if (tid < 3) {
        if (tid < sg.shift) rb[tid] = -INFINITY;
      } else if (tid < 6) {
        const int pz = sg.shift + V + (tid - 3);
        if (pz <= V + 2) rb[pz] = -INFINITY;
      }
      csync();
      C4S_TR(j, 1);
      if (S.abort_row) {
        if (tid == 0) mbar_wait_bounded(&S.bar, phase ^ 1u);   // let the copy drain (bounded)
        lost0 = row;
        lost1 = next;
        break;
      }
      float* srow = rb + sg.shift;
      if (pen) {
        // repetition penalty (sampling.cpp:19-28), each distinct in-range id once
        const float pv = P.repetition_penalty;
        const float rpen = __frcp_rn(pv);
        if (!longh) {
          // read every id's logit, then write its penalised value: ids that
          // repeat write the same value, so no de-duplication is needed
          float orig[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) orig[q] = (unsigned)hid[q] < (unsigned)V ? srow[hid[q]] : 0.0f;
          csync();
          unsigned redo = 0u;                       // quotients div_rn_try could not prove
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            if ((unsigned)hid[q] < (unsigned)V) {
              const float s = orig[q];
              bool ok = true;
              const float y = (s < 0.0f) ? __fmul_rn(s, pv) : div_rn_try(s, pv, rpen, ok);
              if (ok) srow[hid[q]] = y;
              else redo |= 1u << q;
            }
          }
          for (; redo; redo &= redo - 1u) {
            const int q = __ffs(redo) - 1;
            srow[hid[q]] = div_call(orig[q], pv);
          }
        } else {
          csync();                                 // the bitmap is clear
          auto apply = [&](int t) {
            if ((unsigned)t < (unsigned)V) {
              const unsigned bit = 1u << (t & 31);
              if (!(atomicOr(&bm[t >> 5], bit) & bit)) {
                const float s = srow[t];
                srow[t] = (s < 0.0f) ? __fmul_rn(s, pv) : div_rn(s, pv, rpen);
              }
            }
          };
#pragma unroll
          for (int q = 0; q < 8; ++q) apply(hid[q]);
          for (long long jj = h0 + tid + (long long)F_HIST_WORDS; jj < h1; jj += NT) apply(a.hist[jj]);
        }
        csync();
      }
      C4S_TR(j, 2);
      const FGeo g = fgeo(V, sg.shift);
      int fr;
      if constexpr (INL) fr = f_row_body<true>(sa, row, cur, rb, g, S, L);
      else fr = f_row(sa, row, cur, rb, g, S, L);
      if (fr == F_GENERAL) {
        C4S_TR_INFO(j, 3);
        csync();
        if (!general_row(sa, row, reinterpret_cast<float*>(fsm + GL.row), reinterpret_cast<unsigned*>(fsm + GL.bitmap),
                         reinterpret_cast<unsigned*>(fsm + GL.cnt),
                         reinterpret_cast<unsigned long long*>(fsm + GL.mass),
                         reinterpret_cast<unsigned long long*>(fsm + GL.key), reinterpret_cast<double*>(fsm + GL.pv),
                         GS, gphase)) {
          lost0 = row;
          lost1 = next;
          break;
        }
        fill_ninf();                               // the general layout overwrote the row buffer
      }
    } else if (tid == 0) {
      a.out_ids[row] = -1;
    }
    if (tid == 0)                                   // the row after next
      S.nrow[(j + 1) & 1] = next >= a.B ? a.B : tickets ? G + (int)atomicAdd(&ctr[0], 1u) : next + 1;
    cp_async_wait<0>();
    csync();                                       // next metadata visible; the row buffer is free
    sg = Staged{0, 0, -1, 0.0f};
    if (next < a.B && nxt.active) sg = stage_row(a.logits + (long long)next * a.ld, V, rb, &S.bar);
    C4S_TR(j, 7);
    row = next;
  }
  // a CTA that stopped (a bounded wait gave up, C4S_DEVERR_TIMEOUT) marks
  // the rows it held as not sampled; the other CTAs take the rest
  cp_async_wait<0>();
  csync();
  if (tid == 0) {
    if (lost0 < a.B) a.out_ids[lost0] = -1;
    if (lost1 < a.B) a.out_ids[lost1] = -1;
  }
  // the last CTA clears the ticket counters for the next launch
  if (tid == 0 && tickets) {
    __threadfence();
    if (atomicAdd(&ctr[1], 1u) == (unsigned)G - 1u) {
      ctr[0] = 0u;
      ctr[1] = 0u;
    }
  }
}

// the batched form (B > 2 SMs), the small-batch form (B <= SMs) and between
// them two CTAs per SM with the common path inlined (128 registers)
constexpr int FUSED_MINB = 3;
inline constexpr auto fused_kernel = fused_kernel_t<FUSED_MINB, false>;
inline constexpr auto fused_small_kernel = fused_kernel_t<1, true>;
inline constexpr auto fused_mid_kernel = fused_kernel_t<2, true>;

}  // namespace c4s
