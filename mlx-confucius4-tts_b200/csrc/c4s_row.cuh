// c4s_row.cuh -- the row kernel of the fast sampling path (sm_100a).
//
// One CTA of RT = 128 threads works one row at a time, five CTAs per SM. The
// row is staged whole into shared memory by one bulk-async copy (the TMA
// engine; an mbarrier with a bounded wait), and every pass reads it from
// there with 16-byte loads: warp w owns a contiguous segment of the row's
// 16-byte slots and lane l its slots l, l+32, ... of that segment, so the
// loads are conflict-free and a warp's elements come in index order (slot,
// then component), which the ordered candidate lists need. No element array
// lives in registers, which keeps the kernel at <= 102 registers: five rows
// in flight per SM hide each other's copy and barrier latencies.
//
// Per row (text2semantic.cpp:303-331 semantics, sampling.cpp:14-76):
//   penalty (sampling.cpp:19-28) in shared memory, each distinct id once;
//   greedy: first index of the maximum (sampling.cpp:73-76);
//   top-k rows: the maxima threshold (see below) selects >= k candidates,
//     written in index order as ckey(fl(x/T), i) for the list kernel, which
//     finishes top-k, top-p and the draw exactly;
//   rows without top-k: an octave histogram of error-bounded estimates of
//     exp(y - m_y) locates the top-p crossing; the octaves down to it (and a
//     little deeper while the list stays short) form the list, the rest an
//     estimated tail with a proven error bound (est_err);
//   everything else (non-finite maxima, |m_y| >= 2^18, min_tokens_to_keep
//   != 1, lists over LCAP, an undecidable crossing octave) goes to the
//   general path (defer_kernel).
#pragma once

namespace c4s {

constexpr int RT = 128;                            // row kernel threads
constexpr int RWARP = RT / 32;
constexpr int R_SLOTS = (F_MAXV + 3 + 3) / 4;      // 16-byte slots of a staged row (shift <= 3)
constexpr int R_Q = ((R_SLOTS + RWARP - 1) / RWARP + 31) / 32;   // slots per lane
constexpr size_t R_SMEM = (size_t)R_SLOTS * 16;
static_assert(R_Q * 32 * RWARP == R_SLOTS, "the warps' segments tile the buffer exactly");
constexpr int HREP = 8;                            // replicas of each warp's octave bins

// CTA barrier of the row kernel (named barrier 2, RT threads), non-aligned
// like csync(): warps may arrive with diverged lanes.
__device__ __forceinline__ void rsync() { asm volatile("barrier.sync 2, %0;" ::"n"(RT) : "memory"); }

struct RShared {
  unsigned long long bar;
  MetaSlot meta[2];
  int nrow[2];
  unsigned bm[(F_MAXV + 31) / 32 + 4];             // penalty de-duplication bitmap
  unsigned hw[RWARP][HREP][33];                    // octave bins, per warp and lane & 7; rows of 33 words
                                                   // put the replicas of a bin in different banks
  unsigned redu[RWARP];
  int redi[RWARP];
  float redf[RWARP];
  int abort_row;
  int ocnt[ROW_CLASSES];                           // rows per cost class (with a.order)
};

// Slot geometry of one row: element i sits at buffer position shift + i;
// warp w owns slots [w seg, (w+1) seg), seg a multiple of 32 with 4 seg <=
// R_SLOTS, and every buffer position outside the row holds -inf (the kernel
// fills the buffer once and clears the few positions each row's shift
// exposes), so passes read whole segments without bounds checks.
struct RGeo {
  int V, shift, nq, seg;
};
__device__ __forceinline__ RGeo rgeo(int V, int shift) {
  RGeo g;
  g.V = V;
  g.shift = shift;
  const int nslot = (V + shift + 3) >> 2;
  g.seg = (((nslot + RWARP - 1) / RWARP) + 31) & ~31;
  g.nq = g.seg >> 5;
  return g;
}
// Slot of this lane's q-th load (q < g.nq).
__device__ __forceinline__ int rslot(const RGeo& g, int q) {
  return (threadIdx.x >> 5) * g.seg + 32 * q + (threadIdx.x & 31);
}
__device__ __forceinline__ float4 rload(const float* rb, const RGeo& g, int f) {
  return reinterpret_cast<const float4*>(rb)[f];
}
__device__ __forceinline__ float f4c(const float4& v, int c) { return c == 0 ? v.x : c == 1 ? v.y : c == 2 ? v.z : v.w; }

// Count of set bits of `m` (4 bits per lane) below this lane, and the warp
// total, from three ballots.
__device__ __forceinline__ int warp_prefix4(int nl, int* tot) {
  const unsigned lt = (1u << (threadIdx.x & 31)) - 1u;
  const unsigned b0 = __ballot_sync(FULL, nl & 1), b1 = __ballot_sync(FULL, nl & 2), b2 = __ballot_sync(FULL, nl & 4);
  *tot = __popc(b0) + 2 * __popc(b1) + 4 * __popc(b2);
  return __popc(b0 & lt) + 2 * __popc(b1 & lt) + 4 * __popc(b2 & lt);
}

// Writes ckey(x, i) of the elements selected by `sel` (penalised, untempered
// values: the list kernel tempers them) in index order, starting at
// keys[base] for this warp. Whole warp calls.
template <typename Sel>
__device__ __forceinline__ void write_list(unsigned long long* keys, int base, const float* rb, const RGeo& g,
                                           Sel sel) {
  int run = base;
#pragma unroll 2
  for (int q = 0; q < g.nq; ++q) {
    const int f = rslot(g, q);
    const float4 v = rload(rb, g, f);
    const int m = (sel(v.x) ? 1 : 0) | (sel(v.y) ? 2 : 0) | (sel(v.z) ? 4 : 0) | (sel(v.w) ? 8 : 0);
    if (__any_sync(FULL, m)) {
      int tot;
      int pos = run + warp_prefix4(__popc(m), &tot);
      const int i0 = 4 * f - g.shift;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (m & (1 << c)) keys[pos++] = ckey(f4c(v, c), i0 + c);
      run += tot;
    }
  }
}

// Block sum of per-thread counts: every thread gets its warp's base and the total.
__device__ __forceinline__ int rblock_base(int cnt, RShared& S, int* total) {
  const int w = threadIdx.x >> 5;
  const int ws = __reduce_add_sync(FULL, cnt);
  if ((threadIdx.x & 31) == 0) S.redi[w] = ws;
  rsync();
  int base = 0, t = 0;
#pragma unroll
  for (int k = 0; k < RWARP; ++k) {
    if (k < w) base += S.redi[k];
    t += S.redi[k];
  }
  rsync();
  *total = t;
  return base;
}

// Octave of an element without top-k: b(x) = min(trunc(-t log2 e), NOCT) for
// t = RN(x RN(1/T) - m_y), the one-FMA estimate of y - m_y. Every step is
// monotone in x, so the elements in octaves <= bl are exactly those >= some
// x*, and the list and its tail are separated by one comparison. An element
// in octave b < NOCT has |t| < (b+1) ln 2, as oct_d() assumes.
__device__ __forceinline__ float oct_t(const RowCtx& rc, float x) { return fmaf(x, rc.rT, -rc.m_y); }
__device__ __forceinline__ int oct_of_t(float t) { return (int)fminf(t * -1.4426950408889634f, (float)NOCT); }

// The smallest x with oct(x) <= bl (it exists: oct(m_x) = 0), by bisection
// over the float order between -inf (octave NOCT > bl) and m_x.
__device__ __forceinline__ float list_threshold(const RowCtx& rc, int bl) {
  unsigned lo = fkey(-INFINITY), hi = fkey(rc.m_x);
  while (hi - lo > 1u) {
    const unsigned mid = lo + ((hi - lo) >> 1);
    if (oct_of_t(oct_t(rc, fkey_inv(mid))) <= bl) hi = mid;
    else lo = mid;
  }
  return fkey_inv(hi);
}

__device__ __forceinline__ void defer_to_general(const Args& a, int row) {
  if (threadIdx.x == 0) {
    a.jobs[row].kind = JOB_DEFER;
    defer_row(a, row);
  }
}

// The processed row (what the reference's vector holds before top-k/top-p
// masking, which the mask kernel applies afterwards).
__device__ __noinline__ void write_row_smem(const Args& a, const float* rb, const RGeo g, const RowCtx rc,
                                            bool temper) {
  float* o = a.out_logits + (long long)rc.row * a.out_ld;
  for (int q = 0; q < g.nq; ++q) {
    const int f = rslot(g, q);
    const float4 v = rload(rb, g, f);
    const int i0 = 4 * f - g.shift;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int i = i0 + c;
      if ((unsigned)i < (unsigned)g.V) o[i] = temper ? yex(rc, f4c(v, c)) : f4c(v, c);
    }
  }
}

// A top-k row, out of line like rows without top-k.
__device__ __noinline__ int topk_body(const Args& a, int row, const RowCtx rc, const float* rb, const RGeo g,
                                      RShared& S, unsigned long long* keys, int k, bool two, float tm, float t2) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // ---- top-k rows: candidates >= the maxima threshold form the list ----
  // a warp whose kw-th largest lane maximum (of the two largest per lane
  // when `two`) is finite has >= kw elements >= it, so >= k elements are >=
  // tau, the smallest over the warps (-inf: not enough elements; general path)
  if (k > RT * (two ? 2 : 1)) return ROW_GENERAL;
  const float tau = u_threshold<RT>(tm, t2, two, rc.m_x, k, &S.hw[0][0][0], &S.redu[0], [] { rsync(); }, true);
  // fl(x/T) merges x only with values at most |x| 2^-23 below it: lowering tau
  // by 2^-18 relative (+ 2^-18 absolute) keeps every x tied with tau after /T
  const float tau_lo = tau - (fabsf(tau) + 1.0f) * 3.814697265625e-06f;
  if (!(tau_lo > -INFINITY)) return ROW_GENERAL;
  // one pass: each warp stages its candidates' buffer positions, in index
  // order, in its share of the (here unused) octave-bin area; once the warps'
  // counts give their list offsets it copies them out (a warp with more
  // candidates than fit writes its list with a second pass instead)
  unsigned short* stage = reinterpret_cast<unsigned short*>(&S.hw[warp][0][0]);
  constexpr int STAGE_CAP = HREP * 32 * 2;
  int run = 0;
#pragma unroll 2
  for (int q = 0; q < g.nq; ++q) {
    const int f = rslot(g, q);
    const float4 v = rload(rb, g, f);
    const int m = (v.x >= tau_lo ? 1 : 0) | (v.y >= tau_lo ? 2 : 0) | (v.z >= tau_lo ? 4 : 0) | (v.w >= tau_lo ? 8 : 0);
    if (__any_sync(FULL, m)) {
      int tot;
      int pos = run + warp_prefix4(__popc(m), &tot);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (m & (1 << c)) {
          if (pos < STAGE_CAP) stage[pos] = (unsigned short)(4 * f + c);
          ++pos;
        }
      }
      run += tot;
    }
  }
  int ng;
  const int base = rblock_base(lane == 0 ? run : 0, S, &ng);
  if (ng > LCAP) return ROW_GENERAL;
  if (run <= STAGE_CAP) {
    __syncwarp();
    for (int i = lane; i < run; i += 32) {
      const int bp = stage[i];
      keys[base + i] = ckey(rb[bp], bp - g.shift);
    }
  } else {
    write_list(keys, base, rb, g, [&](float x) { return x >= tau_lo; });
  }
  if (tid == 0) {
    RowJob& J = a.jobs[row];
    fill_job(J, rc, JOB_TOPK, ng, k);
    queue_long_list(a, row, ng);
    J.tail = 0.0;
    J.tail_err = 0.0;
    J.ykex = 0u;
  }
  if (a.out_logits) write_row_smem(a, rb, g, rc, true);
  return ROW_DONE;
}

// A row without top-k (top-p over the whole row, sampling.cpp:42-71), out of
// line: the per-row paths stay small enough to share the instruction cache.
__device__ __noinline__ int k0_body(const Args& a, int row, const RowCtx rc, const float* rb, const RGeo g,
                                    RShared& S, unsigned long long* keys) {
  const int V = a.V;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // top_p >= 1 and the forced binned paths: general path
  if (!(rc.thr > 0.0) || (a.debug & C4S_DEBUG_FORCE_BINS)) return ROW_GENERAL;
  // octave histogram of the estimates: per-warp fixed-point bins (exact adds)
  {
#pragma unroll
    for (int r = 0; r < HREP; ++r) S.hw[warp][r][lane] = 0u;
  }
  __syncwarp();
  unsigned* hrep = &S.hw[warp][lane & (HREP - 1)][0];   // fewer lanes per bin address
#pragma unroll 2
  for (int q = 0; q < g.nq; ++q) {
    const float4 v = rload(rb, g, rslot(g, q));
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
  rsync();
  // every warp: lane b holds octave b's mass; suffix sums give the mass below
  // each octave, ballots the crossing octave and the list's last octave
  double o = 0.0;
  if (lane <= NOCT) {
    unsigned long long qs = 0ull;
#pragma unroll
    for (int w = 0; w < RWARP; ++w)
#pragma unroll
      for (int r = 0; r < HREP; ++r) qs += S.hw[w][r][lane];
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
    if (bc < 0 || bc == NOCT) return ROW_GENERAL;
    // the list: octaves 0..bl, bl >= bc the first whose tail is clearly below Th
    const bool okl = lane >= bc && lane < NOCT && blw + 2.0 * est_err(blw, wblw, rc.m_y, 33, V) + rc.thr * es + rnd < Th;
    const unsigned lb = __ballot_sync(FULL, okl);
    bl = lb ? __ffs(lb) - 1 : -1;
    if (bl >= 0) {
      // go deeper while the list stays short, until the tail is below Th/64:
      // the list kernel's decision band (which scales with the tail) then
      // rarely reaches the crossing element
      const unsigned small = __ballot_sync(FULL, lane >= bl && lane < NOCT && blw <= Th * 0.015625);
      const unsigned fits = __ballot_sync(FULL, lane >= bl && lane < NOCT && pre <= 0.5 * LIST_DEEP);
      const int bt = small ? __ffs(small) - 1 : NOCT - 1;
      const int bf = fits ? 31 - __clz(fits) : bl;
      bl = max(bl, min(bt, bf));
    }
  }
  if (bl < 0) return ROW_GENERAL;
  const double nb = __shfl_sync(FULL, pre, bl);
  if (nb > 2.0 * LCAP) return ROW_GENERAL;
  // the list: elements in octaves <= bl, i.e. >= x*, in index order
  const float xs = list_threshold(rc, bl);
  auto in_list = [&](float x) { return x >= xs; };
  // one pass, as for top-k rows: positions staged per warp in the octave-bin
  // area (every warp has read the bins once the barrier is passed), plus the
  // largest element below the list
  rsync();
  unsigned short* stage = reinterpret_cast<unsigned short*>(&S.hw[warp][0][0]);
  constexpr int STAGE_CAP = HREP * 32 * 2;
  int run = 0;
  float xmx = -INFINITY;
#pragma unroll 2
  for (int q = 0; q < g.nq; ++q) {
    const int f = rslot(g, q);
    const float4 v = rload(rb, g, f);
    int m = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float x = f4c(v, c);
      if (in_list(x)) m |= 1 << c;
      else xmx = fmaxf(xmx, x);
    }
    if (__any_sync(FULL, m)) {
      int tot;
      int pos = run + warp_prefix4(__popc(m), &tot);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (m & (1 << c)) {
          if (pos < STAGE_CAP) stage[pos] = (unsigned short)(4 * f + c);
          ++pos;
        }
      }
      run += tot;
    }
  }
  {
    const unsigned km = __reduce_max_sync(FULL, fkey(xmx));
    if (lane == 0) S.redu[warp] = km;
  }
  int ng;
  const int base = rblock_base(lane == 0 ? run : 0, S, &ng);   // its barriers also publish S.redu
  if (ng > LCAP) return ROW_GENERAL;
  unsigned kx = S.redu[0];
#pragma unroll
  for (int w = 1; w < RWARP; ++w) kx = kx > S.redu[w] ? kx : S.redu[w];
  const float xm = fkey_inv(kx);
  if (run <= STAGE_CAP) {
    __syncwarp();
    for (int i = lane; i < run; i += 32) {
      const int bp = stage[i];
      keys[base + i] = ckey(rb[bp], bp - g.shift);
    }
  } else {
    write_list(keys, base, rb, g, in_list);
  }
  const double tl = __shfl_sync(FULL, blw, bl), tl_err = est_err(tl, __shfl_sync(FULL, wblw, bl), rc.m_y, 33, V);
  if (tid == 0) {
    RowJob& J = a.jobs[row];
    fill_job(J, rc, JOB_K0, ng, 0);
    queue_long_list(a, row, ng);
    J.tail = tl;
    J.tail_err = tl_err;
    J.ykex = xm > -INFINITY ? fkey(yex(rc, xm)) : 0u;
  }
  if (a.out_logits) write_row_smem(a, rb, g, rc, true);
  return ROW_DONE;
}

// One staged, penalised row. Returns ROW_DONE or ROW_GENERAL.
__device__ __forceinline__ int row_body(const Args& a, const Args& ao, int row, const MetaSlot& M, const float* rb,
                                         const RGeo& g, RShared& S) {
  const int V = a.V;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const c4s_row_params P = M.P;
  const int k = P.top_k;
  const bool do_k = k > 0 && k < V;
  const bool two = !P.greedy && do_k && k > RWARP * 32 / 2;   // the two largest per lane seed the list

  // ---- row max, per-lane maxima (and second maxima), valid elements per lane ----
  // (top-k rows: the threshold histogram's bins are cleared here, ordered
  // before their use by the barrier of the max reduction; the area's last
  // use, the previous row's staging, ended before the row's barriers)
  if (!P.greedy && do_k)
    for (int i = tid; i < 256; i += RT) (&S.hw[0][0][0])[i] = 0u;
  float tm = -INFINITY, t2 = -INFINITY;
#pragma unroll 4
  for (int q = 0; q < g.nq; ++q) {
    const float4 v = rload(rb, g, rslot(g, q));
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
  rsync();
  unsigned kall = S.redu[0];
#pragma unroll
  for (int w = 1; w < RWARP; ++w) kall = kall > S.redu[w] ? kall : S.redu[w];
  const float m_x = fkey_inv(kall);
  // (S.redu is next written behind later barriers: the greedy path's below,
  // the threshold's result and the no-top-k path's after their own barriers)

  RowCtx rc;
  rc.row = row; rc.V = V; rc.i0 = 0;
  rc.T = P.temperature;
  rc.do_t = !(rc.T == 1.0f || rc.T <= 0.0f);

  // ---- greedy: first index of the max (sampling.cpp:73-76) ----
  if (P.greedy) {
    rsync();                                       // every warp has read S.redu
    unsigned cand = 0xffffffffu;
    if (m_x > -INFINITY && tm == m_x) {
      for (int q = 0; q < g.nq; ++q) {
        const int f = rslot(g, q);
        const float4 v = rload(rb, g, f);
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
    rsync();
    if (tid == 0) {
      unsigned b = S.redu[0];
      for (int w = 1; w < RWARP; ++w) b = S.redu[w] < b ? S.redu[w] : b;
      a.out_ids[row] = b == 0xffffffffu ? 0 : (int)b;
      a.jobs[row].kind = JOB_NONE;
    }
    if (a.out_logits) write_row_smem(ao, rb, g, rc, false);
    rsync();
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
  rc.thr = __dsub_rn(1.0, (double)P.top_p);
  {
    unsigned long long xs = M.rng;
    xs ^= xs << 13; xs ^= xs >> 7; xs ^= xs << 17;
    rc.xs = xs;
    rc.u53 = xs >> 11;
    rc.u = (double)rc.u53 * 1.1102230246251565e-16;   // (x>>11) / 2^53, exact
  }
  unsigned long long* keys = a.lkeys + (size_t)row * LCAP;

  if (do_k) return topk_body(ao, row, rc, rb, g, S, keys, k, two, tm, t2);
  return k0_body(ao, row, rc, rb, g, S, keys);
}

// Rows by cost class for the row kernel, dearest first, so that its last
// wave holds cheap rows and its CTAs finish together: sampled rows without
// top-k (octave histogram), top-k above 64 (two maxima per lane), other top-k,
// then greedy and inactive rows. One thread per row, ORDER_NT rows per CTA:
// class slots from shared-memory counters (one atomic per class and warp),
// then one global atomic per class and CTA reserves the CTA's range of the
// class; the class sizes accumulate in defer_cnt[ORD_CNT + c] (zero at the
// start: cleared by the general kernel of the previous launch sequence).
constexpr int ORDER_NT = 512;
__global__ void __launch_bounds__(ORDER_NT) order_kernel(Args a) {
  __shared__ unsigned cnt[ROW_CLASSES], gbase[ROW_CLASSES];
  const int lane = threadIdx.x & 31;
  if (threadIdx.x < ROW_CLASSES) cnt[threadIdx.x] = 0u;
  __syncthreads();
  const int r = blockIdx.x * ORDER_NT + (int)threadIdx.x;
  int c = -1;
  grid_dep_launch();
  grid_dep_wait();                                 // the previous sequence clears the class counters (and an
                                                   // earlier kernel of the stream may write params or active flags)
  if (r < a.B) {
    const c4s_row_params P = a.params[(long long)r * a.params_stride];
    const bool act = a.active == nullptr || a.active[r] != 0;
    const int k = P.top_k;
    c = (!act || P.greedy) ? 3 : (k <= 0 || k >= a.V) ? 0 : k > RWARP * 32 / 2 ? 1 : 2;
  }
  unsigned slot = 0u;
#pragma unroll
  for (int cc = 0; cc < ROW_CLASSES; ++cc) {
    const unsigned m = __ballot_sync(FULL, c == cc);
    if (m == 0u) continue;
    const int leader = __ffs(m) - 1;
    unsigned base = 0u;
    if (lane == leader) base = atomicAdd(&cnt[cc], (unsigned)__popc(m));
    base = __shfl_sync(FULL, base, leader);
    if (c == cc) slot = base + (unsigned)__popc(m & ((1u << lane) - 1u));
  }
  __syncthreads();
  if (threadIdx.x < ROW_CLASSES)
    gbase[threadIdx.x] = cnt[threadIdx.x] ? atomicAdd(&a.defer_cnt[ORD_CNT + threadIdx.x], cnt[threadIdx.x]) : 0u;
  __syncthreads();
  if (c >= 0) {
    const unsigned s = gbase[c] + slot;
    if (s < (unsigned)a.chunk) a.order[(size_t)c * a.chunk + s] = r;
  }
}

// The row of the row kernel's t-th ticket (B: none left).
__device__ __forceinline__ int ticket_row(const Args& a, const RShared& S, int t) {
  if (t >= a.B) return a.B;
  if (a.order == nullptr) return t;
#pragma unroll
  for (int c = 0; c < ROW_CLASSES; ++c) {
    if (t < S.ocnt[c]) return t < a.chunk ? a.order[(size_t)c * a.chunk + t] : a.B;
    t -= S.ocnt[c];
  }
  return a.B;
}

// Persistent row kernel: rows handed out dynamically (the first G statically).
__global__ void __launch_bounds__(RT, 5) row_kernel(Args a) {
  extern __shared__ __align__(128) float rb[];     // the staged row
  __shared__ RShared S;
  // the out-of-line paths read the arguments from here: a reference to the
  // kernel parameter would give every thread a copy in local memory
  __shared__ Args sa;
  const int V = a.V;
  const int tid = threadIdx.x;
  const int G = gridDim.x;
  const int nbm = (V + 31) / 32;

  if (tid == 0) {
    mbar_init(&S.bar, 1);
    sa = a;
  }
  // every buffer position outside a row reads as -inf (see RGeo)
  for (int i = tid; i < 4 * R_SLOTS; i += RT) rb[i] = -INFINITY;
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
  unsigned* row_ctr = a.defer_cnt + 2;
  grid_dep_launch();
  grid_dep_wait();                                 // counters, order and RNG states of earlier launches
  if (a.order != nullptr) {
    if (tid < ROW_CLASSES) S.ocnt[tid] = (int)a.defer_cnt[ORD_CNT + tid];
    rsync();
  }
  const int r0 = ticket_row(a, S, blockIdx.x);
  if (tid == 0) S.nrow[0] = ticket_row(a, S, G + (int)atomicAdd(row_ctr, 1u));
  issue_meta(r0, S.meta[0]);
  cp_async_commit();
  if (tid == 6 && r0 < a.B) S.meta[0].active = act_pend;
  cp_async_wait<0>();
  rsync();
  unsigned phase = 0;
  Staged sg{0, 0, -1, 0.0f};
  if (r0 < a.B && S.meta[0].active) sg = stage_row(a.logits + (long long)r0 * a.ld, V, rb, &S.bar);

  int j = 0;
  for (int row = r0; row < a.B; ++j) {
    const MetaSlot& cur = S.meta[j & 1];
    MetaSlot& nxt = S.meta[(j + 1) & 1];
    const int next = S.nrow[j & 1];
    issue_meta(next, nxt);
    cp_async_commit();
    if (tid == 32 && next < a.B) prefetch_row(a.logits + (long long)next * a.ld, V);
    if (tid == 6 && next < a.B) nxt.active = act_pend;
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
      // histories beyond the ids the threads hold in registers de-duplicate through a bitmap
      const bool longh = h1 - h0 > 16LL * RT;
      if (longh)
        for (int w = tid; w < nbm; w += RT) S.bm[w] = 0u;
      // the first 16 ids per thread in flight while the row arrives
      int hid[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        const long long jj = h0 + tid + (long long)q * RT;
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
      rsync();
      if (S.abort_row) {
        if (tid == 0) mbar_wait_bounded(&S.bar, phase ^ 1u);   // let the copy drain (bounded)
        break;
      }
      float* srow = rb + sg.shift;
      if (pen) {
        // repetition penalty (sampling.cpp:19-28): each distinct in-range id once
        const float pv = P.repetition_penalty;
        const float rpen = __frcp_rn(pv);
        auto apply = [&](int t) {
          if ((unsigned)t < (unsigned)V) {
            const unsigned bit = 1u << (t & 31);
            const unsigned old = atomicOr(&S.bm[t >> 5], bit);
            if (!(old & bit)) {
              const float s = srow[t];
              srow[t] = (s < 0.0f) ? __fmul_rn(s, pv) : div_rn(s, pv, rpen);
            }
          }
        };
        if (!longh) {
          // every id reads its logit, a barrier, every id writes the
          // penalised value: ids that repeat write the same value, so no
          // de-duplication (bitmap, atomics) is needed
          float orig[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) orig[q] = (unsigned)hid[q] < (unsigned)V ? srow[hid[q]] : 0.0f;
          rsync();
          unsigned redo = 0u;                       // quotients div_rn_try could not prove
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            if ((unsigned)hid[q] < (unsigned)V) {
              const float sv = orig[q];
              bool ok = true;
              const float y = (sv < 0.0f) ? __fmul_rn(sv, pv) : div_rn_try(sv, pv, rpen, ok);
              if (ok) srow[hid[q]] = y;
              else redo |= 1u << q;
            }
          }
          for (; redo; redo &= redo - 1u) {
            const int q = __ffs(redo) - 1;
            srow[hid[q]] = div_call(orig[q], pv);
          }
        } else {
          // claim the ids first (independent atomics in flight together),
          // then penalise the ones this thread claimed first
          unsigned first = 0u;
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const int t = hid[q];
            if ((unsigned)t < (unsigned)V) {
              const unsigned bit = 1u << (t & 31);
              if (!(atomicOr(&S.bm[t >> 5], bit) & bit)) first |= 1u << q;
            }
          }
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            if (first & (1u << q)) {
              const int t = hid[q];
              const float sv = srow[t];
              srow[t] = (sv < 0.0f) ? __fmul_rn(sv, pv) : div_rn(sv, pv, rpen);
            }
          }
          for (long long jj = h0 + tid + 16LL * RT; jj < h1; jj += RT) apply(a.hist[jj]);
        }
        rsync();
      }
      const RGeo g = rgeo(V, sg.shift);
      if (row_body(a, sa, row, cur, rb, g, S) == ROW_GENERAL) defer_to_general(a, row);
    } else if (tid == 0) {
      a.out_ids[row] = -1;
      a.jobs[row].kind = JOB_NONE;
    }
    if (tid == 0) S.nrow[(j + 1) & 1] = next < a.B ? ticket_row(a, S, G + (int)atomicAdd(row_ctr, 1u)) : a.B;   // the row after next
    cp_async_wait<0>();
    rsync();                                       // next metadata visible; the row buffer is free
    sg = Staged{0, 0, -1, 0.0f};
    if (next < a.B && nxt.active) sg = stage_row(a.logits + (long long)next * a.ld, V, rb, &S.bar);
    row = next;
  }
}

}  // namespace c4s
