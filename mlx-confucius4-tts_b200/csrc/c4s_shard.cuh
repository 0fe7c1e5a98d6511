// c4s_shard.cuh -- vocab-sharded sampling (a row's vocabulary split into
// contiguous shards, one per GPU).
//
// The reference samples one whole row on the host (text2semantic.cpp:303-331:
// repetition_penalty, temperature, top_k, top_p, draw). When the vocabulary is
// split across GPUs no GPU holds a whole row, so the step runs in two stages
// with an all-gather of a few candidates between them:
//
//   shard_kernel  (every shard, its own columns): penalty over the history ids
//                 that fall in the shard (sampling.cpp:19-28), temperature
//                 (sampling.cpp:14-17; sampled rows only), then the shard's 64
//                 largest values, ties at the 64th broken by ascending index,
//                 written as (value, global index) pairs, largest first;
//   merge_kernel  (after the gather, on the candidates of all shards): greedy
//                 argmax (sampling.cpp:73-76), or top_k (sampling.cpp:30-40),
//                 top_p (sampling.cpp:42-71) and the xorshift64 draw
//                 (text2semantic.cpp:150-165) over the candidates.
//
// Exactness. For 1 <= top_k <= 64 the global top_k threshold is the k-th
// largest candidate (every element of the global k largest is among its
// shard's 64 largest), and every element that survives top_k is a candidate
// unless a shard has more than 64 elements equal to its 64th value and that
// value is the threshold; the shard flags that case (C4S_CAND_TIES on its
// last entry) and the merge reports it (C4S_DEVERR_SHARD) instead of guessing.
// Elements outside the candidates are -inf after top_k: they add exact zeros
// to the reference's double sums (ascending-value order for top_p, index
// order for the draw), so summing the candidates alone in the same orders
// gives the same doubles. The only position-dependent case is a draw with
// r == 0 (xorshift output below 2^11), where the reference returns index 0.
#pragma once

namespace c4s {

constexpr int SHARD_CAND = C4S_SHARD_CANDIDATES;  // candidates per row and shard
constexpr int SHARD_LIST = 1024;                   // fast-path list capacity
constexpr int MAX_SHARDS = C4S_MAX_SHARDS;
constexpr unsigned CAND_TIES = C4S_CAND_TIES;
static_assert(SHARD_CAND * MAX_SHARDS % NT == 0, "merge ranks whole passes of the block");

struct ShardArgs {
  const float* logits;   // row r at logits + r * ld: G == 1 one shard's columns;
                         // G > 1 the columns Vtot split into G shards (shard_span(s))
  int B, Vs;             // rows; shard width (G > 1: the widest shard)
  long long ld;
  int voff, Vtot;        // global index of column 0; G > 1: the width that is split
  int G;                 // shards worked by this launch (1, or all of the given columns)
  long long cand_stride; // G > 1: candidates between the shards' blocks
  const int* hist;
  const long long* hist_off;
  long long hist_total;
  const c4s_row_params* params;
  int params_stride;
  const unsigned char* active;
  c4s_candidate* cand;   // [B][SHARD_CAND] (G > 1: [G][cand_stride])
  unsigned* errflags;
};

// Columns [off, off + width) of shard s when V columns are split into G
// contiguous shards whose widths differ by at most one.
__host__ __device__ inline void shard_span(int V, int G, int s, int& off, int& width) {
  const int base = V / G, extra = V % G;
  off = s * base + (s < extra ? s : extra);
  width = base + (s < extra ? 1 : 0);
}

struct MergeArgs {
  const c4s_candidate* cand;  // shard s, row r: cand + s * shard_stride + r * SHARD_CAND
  int G, B, Vtot;
  long long shard_stride;
  const c4s_row_params* params;
  int params_stride;
  unsigned long long* rng;
  const unsigned char* active;
  int* out_ids;
  unsigned* errflags;
};

__host__ __device__ inline size_t shard_smem_bytes(int Vs) {
  return (size_t)SHARD_LIST * 8 + align_up((size_t)Vs, 4) * 4 + (size_t)((Vs + 31) / 32) * 4;
}

// Writes the row's 64 candidates from an ascending list of keys
// (~fkey(value) << 32 | local index; value already tempered): largest value
// first, ties by index.
__device__ __forceinline__ void shard_emit(c4s_candidate* out, int voff, const unsigned long long* list,
                                           bool ties) {
  const int t = threadIdx.x;
  if (t < SHARD_CAND) {
    const unsigned long long k = list[t];
    unsigned gi = (unsigned)(voff + (int)(unsigned)(k & 0xffffffffull));
    if (t == SHARD_CAND - 1 && ties) gi |= CAND_TIES;
    c4s_candidate c;
    c.value = fkey_inv(~(unsigned)(k >> 32));
    c.index = (int)gi;
    out[t] = c;
  }
}

// Eight 16-byte slots of the staged row per thread: slot (ch * 8 + q) * NT +
// tid; slots past the row read as -inf.
constexpr int SHARD_SQ = 8;
__device__ __forceinline__ void shard_slots(float4 (&v)[SHARD_SQ], const float4* s4, int ch, int nv) {
#pragma unroll
  for (int q = 0; q < SHARD_SQ; ++q) {
    const int f = (ch * SHARD_SQ + q) * NT + (int)threadIdx.x;
    v[q] = f < nv ? s4[f] : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
  }
}

__global__ void __launch_bounds__(NT, 3) shard_kernel(ShardArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned long long* list = reinterpret_cast<unsigned long long*>(smem);
  float* srow = reinterpret_cast<float*>(smem + (size_t)SHARD_LIST * 8);
  unsigned* bitmap = reinterpret_cast<unsigned*>(srow + align_up((size_t)a.Vs, 4));  // a.Vs: widest shard
  __shared__ unsigned s_wk[NWARP];
  __shared__ unsigned s_hist[256];
  __shared__ float s_mx[NWARP];
  __shared__ int s_scan[NWARP];
  __shared__ unsigned s_res;
  __shared__ int s_cnt, s_digit, s_want;
  static_assert(NT == 256, "one histogram bin per thread");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const long long items = (long long)a.B * a.G;
  for (long long item = blockIdx.x; item < items; item += gridDim.x) {
    if (tid == 0 && item + gridDim.x < items) {  // the next item's columns into L2 (its aligned interior)
      const long long nx = item + gridDim.x;
      const int nrow = (int)(nx / a.G);
      int nl = 0, nw = a.Vs;
      if (a.G > 1) shard_span(a.Vtot, a.G, (int)(nx % a.G), nl, nw);
      const uintptr_t p0 = (uintptr_t)(a.logits + (long long)nrow * a.ld + nl);
      const uintptr_t b0 = (p0 + 15) & ~(uintptr_t)15, b1 = (p0 + (uintptr_t)nw * 4) & ~(uintptr_t)15;
      if (b1 > b0) bulk_prefetch_l2((const void*)b0, (unsigned)(b1 - b0));
    }
    const int row = (int)(item / a.G), sh = (int)(item % a.G);
    if (a.active && !a.active[row]) continue;
    int voff = a.voff, Vs = a.Vs, loff = 0;       // loff: the shard's first column in the given ones
    if (a.G > 1) {
      shard_span(a.Vtot, a.G, sh, loff, Vs);
      voff += loff;
    }
    c4s_candidate* out = a.cand + (long long)sh * a.cand_stride + (long long)row * SHARD_CAND;
    const c4s_row_params P = a.params[(long long)row * a.params_stride];
    const float* g = a.logits + (long long)row * a.ld + loff;
    // 1. stage the shard's row (16-byte loads when the row is aligned), with
    //    the row's history ids loaded while the first eight slots are in flight
    const bool al = (((uintptr_t)g) & 15) == 0;
    const float4* g4 = reinterpret_cast<const float4*>(g);
    float4* s4w = reinterpret_cast<float4*>(srow);
    const int n4 = al ? Vs >> 2 : 0;
    float4 r[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int i = q * NT + tid;
      if (i < n4) r[q] = __ldg(g4 + i);
    }
    // 2. repetition penalty over the history ids inside this shard: up to
    //    HR ids per thread in registers (read-then-write below), longer
    //    histories through a de-duplication bitmap
    constexpr int HR = 4;
    const bool pen = P.repetition_penalty != 1.0f && a.hist_off != nullptr;
    long long h0 = 0, h1 = 0;
    if (pen) {
      h0 = a.hist_off[row];
      h1 = a.hist_off[row + 1];
      if (h0 < 0 || h1 < h0 || h1 > a.hist_total) {
        if (tid == 0) atomicOr(a.errflags, C4S_DEVERR_HIST_RANGE);
        h0 = h1 = 0;
      }
    }
    const bool hshort = h1 - h0 <= (long long)HR * NT;
    int hid[HR];
#pragma unroll
    for (int q = 0; q < HR; ++q) {
      const long long j = h0 + tid + (long long)q * NT;
      hid[q] = (pen && hshort && j < h1) ? __ldg(a.hist + j) : -1;
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int i = q * NT + tid;
      if (i < n4) s4w[i] = r[q];
    }
    for (int i0 = 8 * NT; i0 < n4; i0 += 8 * NT) {  // wider shards: eight 16-byte loads in flight per thread
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int i = i0 + q * NT + tid;
        if (i < n4) r[q] = __ldg(g4 + i);
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int i = i0 + q * NT + tid;
        if (i < n4) s4w[i] = r[q];
      }
    }
    for (int i = 4 * n4 + tid; i < Vs; i += NT) srow[i] = __ldg(g + i);
    if (tid < ((4 - (Vs & 3)) & 3)) srow[Vs + tid] = -INFINITY;
    if (pen && !hshort)
      for (int i = tid; i < (Vs + 31) / 32; i += NT) bitmap[i] = 0u;
    s_hist[tid] = 0u;  // the threshold's bins
    __syncthreads();
    if (pen) {
      const float pv = P.repetition_penalty;
      const float rpv = __frcp_rn(pv);
      if (hshort) {
        // every id inside the shard reads its value, a barrier, every one
        // writes the penalised value: repeated ids write the same value
        float pen_v[HR];
        unsigned pen_u[HR];
#pragma unroll
        for (int q = 0; q < HR; ++q) {
          pen_u[q] = (unsigned)hid[q] - (unsigned)voff;
          if (hid[q] >= 0 && pen_u[q] < (unsigned)Vs) {
            const float s = srow[pen_u[q]];
            pen_v[q] = (s < 0.0f) ? __fmul_rn(s, pv) : div_rn(s, pv, rpv);
          } else {
            pen_u[q] = 0xffffffffu;
          }
        }
        __syncthreads();
#pragma unroll
        for (int q = 0; q < HR; ++q)
          if (pen_u[q] != 0xffffffffu) srow[pen_u[q]] = pen_v[q];
      } else {
        for (long long j = h0 + tid; j < h1; j += NT) {
          const int t = a.hist[j];
          const unsigned u = (unsigned)t - (unsigned)voff;
          if (t >= 0 && u < (unsigned)Vs) {
            const unsigned bit = 1u << (u & 31);
            const unsigned old = atomicOr(&bitmap[u >> 5], bit);
            if (!(old & bit)) {
              const float s = srow[u];
              srow[u] = (s < 0.0f) ? __fmul_rn(s, pv) : div_rn(s, pv, rpv);
            }
          }
        }
      }
      __syncthreads();
    }
    // 3. each thread's two largest penalised values and the row's maximum
    //    (eight 16-byte slots per thread and pass, held in registers; the
    //    buffer's padding to a multiple of 4 holds -inf)
    const bool temper = !P.greedy && !(P.temperature == 1.0f || P.temperature <= 0.0f);
    const float T = P.temperature;
    const int nv = (Vs + 3) >> 2;
    const float4* s4 = reinterpret_cast<const float4*>(srow);
    const int nch = (nv + SHARD_SQ * NT - 1) / (SHARD_SQ * NT);
    float4 v[SHARD_SQ];
    float tm = -INFINITY, t2 = -INFINITY;
    for (int ch = 0; ch < nch; ++ch) {
      shard_slots(v, s4, ch, nv);
#pragma unroll
      for (int q = 0; q < SHARD_SQ; ++q) {
        const float e[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          t2 = fmaxf(t2, fminf(tm, e[c]));
          tm = fmaxf(tm, e[c]);
        }
      }
    }
    const float m_x = block_reduce(tm, MaxF{}, s_mx);
    // 4. a lower bound on the 64th largest value: the 64th largest of the
    //    threads' two largest values (distinct elements), located in a
    //    histogram of key distances from the maximum, so at least 64 elements
    //    are >= tau and few more. Lowered by 2^-18 relative when tempering:
    //    RN(x / T) merges x only with values at most |x| 2^-23 below it, so the
    //    list keeps the elements that may temper to a listed value.
    const float tau = u_threshold<NT>(tm, t2, true, m_x, SHARD_CAND, s_hist, &s_res, [] { csync(); }, true);
    const float bound = temper ? tau - (fabsf(tau) + 1.0f) * 3.814697265625e-06f : tau;
    // 5. every element >= the bound into the list at its thread's offset (a
    //    count, a CTA-wide scan, a write), as untempered value bits << 32 |
    //    local index. One pass of slots (Vs <= 8 * 4 * NT) with a finite
    //    bound: a mask of the thread's elements >= the bound (bit 4q + c:
    //    element 4 (q NT + tid) + c; the -inf padding never counts), the write
    //    visits its set bits only.
    int n0 = 0;
    if (nch == 1 && bound > -INFINITY) {
      shard_slots(v, s4, 0, nv);
      unsigned m = 0u;
#pragma unroll
      for (int q = 0; q < SHARD_SQ; ++q) {
        m |= (v[q].x >= bound ? 1u : 0u) << (4 * q);
        m |= (v[q].y >= bound ? 2u : 0u) << (4 * q);
        m |= (v[q].z >= bound ? 4u : 0u) << (4 * q);
        m |= (v[q].w >= bound ? 8u : 0u) << (4 * q);
      }
      int pos = block_exscan_i32(__popc(m), s_scan, &n0);
      if (n0 <= SHARD_LIST) {
        while (m) {
          const int b = __ffs(m) - 1;
          m &= m - 1u;
          const int idx = 4 * ((b >> 2) * NT + tid) + (b & 3);
          list[pos++] = ((unsigned long long)__float_as_uint(srow[idx]) << 32) | (unsigned)idx;
        }
      }
    } else {
      int cnt = 0;
#pragma unroll 4
      for (int f = tid; f < nv; f += NT) {
        const float4 w = s4[f];
        const int i0 = 4 * f;
        cnt += (w.x >= bound) + (i0 + 1 < Vs && w.y >= bound) + (i0 + 2 < Vs && w.z >= bound) +
               (i0 + 3 < Vs && w.w >= bound);
      }
      int pos = block_exscan_i32(cnt, s_scan, &n0);
      if (n0 <= SHARD_LIST && cnt > 0) {
        for (int f = tid; f < nv; f += NT) {
          const float4 w = s4[f];
          if (fmaxf(fmaxf(w.x, w.y), fmaxf(w.z, w.w)) >= bound) {
            const float e[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int c = 0; c < 4; ++c)
              if (4 * f + c < Vs && e[c] >= bound)
                list[pos++] = ((unsigned long long)__float_as_uint(e[c]) << 32) | (unsigned)(4 * f + c);
          }
        }
      }
    }
    __syncthreads();
    // the key of a list entry: ~fkey(tempered value) << 32 | local index
    auto tkey = [&](unsigned long long raw) {
      const float x = __uint_as_float((unsigned)(raw >> 32));
      const float tv = temper ? __fdiv_rn(x, T) : x;
      return ((unsigned long long)(~fkey(tv)) << 32) | (raw & 0xffffffffull);
    };
    bool fast = n0 >= SHARD_CAND && n0 <= SHARD_LIST;
    if (fast) {
      if (n0 <= NT) {
        // rank sort (keys are distinct): the 65 smallest keys into list[0..64]
        unsigned long long kt = 0ull;
        int r = SHARD_LIST;
        if (tid < n0) {
          kt = tkey(list[tid]);
          list[tid] = kt;
        }
        __syncthreads();
        if (tid < n0) {
          r = 0;
          const ulonglong2* l2 = reinterpret_cast<const ulonglong2*>(list);  // two keys per load
#pragma unroll 4
          for (int j = 0; j < (n0 >> 1); ++j) {
            const ulonglong2 kk = l2[j];
            r += (kk.x < kt) + (kk.y < kt);
          }
          if (n0 & 1) r += list[n0 - 1] < kt;
        }
        __syncthreads();
        if (r <= SHARD_CAND) list[r] = kt;
        __syncthreads();
      } else {
        const int n2 = next_pow2(n0);
        for (int i = tid; i < n2; i += NT) list[i] = i < n0 ? tkey(list[i]) : KEY_MAX;
        __syncthreads();
        bitonic_sort_u64(list, n2);
      }
      if (temper) {
        // every element below the bound tempers to at most RN(prev(bound) / T)
        const float t64 = fkey_inv(~(unsigned)(list[SHARD_CAND - 1] >> 32));
        fast = t64 > __fdiv_rn(nextafterf(bound, -INFINITY), T);
      }
    }
    if (fast) {
      const bool ties = n0 > SHARD_CAND && (list[SHARD_CAND] >> 32) == (list[SHARD_CAND - 1] >> 32);
      shard_emit(out, voff, list, ties);
    } else {
      if (temper) {
        for (int i = tid; i < Vs; i += NT) srow[i] = __fdiv_rn(srow[i], T);
        __syncthreads();
      }
      // Rare (many equal values near the top): exact 64th largest key by a
      // byte-wise radix select, then the larger elements and the first
      // equal ones in index order.
      unsigned prefix = 0u, mask = 0u;
      int want = SHARD_CAND;
      for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += NT) s_hist[i] = 0u;
        __syncthreads();
        for (int i = tid; i < Vs; i += NT) {
          const unsigned k = fkey(srow[i]);
          if ((k & mask) == prefix) atomicAdd(&s_hist[(k >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (warp == 0) {
          unsigned c[8], tot = 0u;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            c[q] = s_hist[255 - 8 * lane - q];
            tot += c[q];
          }
          unsigned inc = tot;
          for (int o = 1; o < 32; o <<= 1) {
            const unsigned y = __shfl_up_sync(FULL, inc, o);
            if (lane >= o) inc += y;
          }
          unsigned acc = inc - tot;
          if (acc < (unsigned)want && (unsigned)want <= inc) {
            for (int q = 0; q < 8; ++q) {
              if (acc + c[q] >= (unsigned)want) {
                s_digit = 255 - 8 * lane - q;
                s_want = want - (int)acc;
                break;
              }
              acc += c[q];
            }
          }
        }
        __syncthreads();
        prefix |= (unsigned)s_digit << shift;
        mask |= 255u << shift;
        want = s_want;
        __syncthreads();
      }
      const unsigned tau = prefix;  // key of the 64th largest; `want` of its copies are needed
      if (tid == 0) s_cnt = 0;
      __syncthreads();
      int eq_before = 0;  // equal elements in earlier chunks (uniform)
      for (int i0 = 0; i0 < Vs; i0 += NT) {
        const int i = i0 + tid;
        const unsigned k = i < Vs ? fkey(srow[i]) : 0u;
        const bool gt = i < Vs && k > tau, eq = i < Vs && k == tau;
        const unsigned mg = __ballot_sync(FULL, gt);
        const unsigned me = __ballot_sync(FULL, eq);
        if (lane == 0) s_wk[warp] = (unsigned)__popc(me);
        __syncthreads();
        int before = eq_before, tot = 0;
#pragma unroll
        for (int w = 0; w < NWARP; ++w) {
          before += w < warp ? (int)s_wk[w] : 0;
          tot += (int)s_wk[w];
        }
        (void)mg;
        const bool take = gt || (eq && before + __popc(me & ((1u << lane) - 1u)) < want);
        if (take) {
          const int pos = atomicAdd(&s_cnt, 1);
          if (pos < SHARD_CAND) list[pos] = ((unsigned long long)(~k) << 32) | (unsigned)i;
        }
        eq_before += tot;
        __syncthreads();
      }
      bitonic_sort_u64(list, SHARD_CAND);
      shard_emit(out, voff, list, eq_before > want);
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(NT) merge_kernel(MergeArgs a) {
  constexpr int NC = SHARD_CAND * MAX_SHARDS;
  __shared__ unsigned long long dk[NC];  // (~fkey(value) << 32) | index: each shard's block ascending
  __shared__ float val[NC];
  __shared__ double pr[NC];
  __shared__ int sv[NC];                 // survivors by descending (value), ascending index
  __shared__ int ord[NC];                // survivors in ascending (value, index) order
  __shared__ unsigned s_tiekey[MAX_SHARDS];
  __shared__ unsigned long long s_red[NWARP];
  __shared__ unsigned s_tk;
  __shared__ int s_m, s_keep, s_bad;
  __shared__ double s_sum;
  const int tid = threadIdx.x;
  const int G = a.G;
  const int n = G * SHARD_CAND;
  for (int row = blockIdx.x; row < a.B; row += gridDim.x) {
    if (a.active && !a.active[row]) {
      if (tid == 0) a.out_ids[row] = -1;
      continue;
    }
    const c4s_row_params P = a.params[(long long)row * a.params_stride];
    unsigned long long best = KEY_MAX;
    for (int j = tid; j < n; j += NT) {
      const int s = j / SHARD_CAND, q = j % SHARD_CAND;
      const c4s_candidate c = a.cand[(long long)s * a.shard_stride + (long long)row * SHARD_CAND + q];
      const unsigned gi = (unsigned)c.index & ~CAND_TIES;
      const unsigned long long d = ((unsigned long long)(~fkey(c.value)) << 32) | gi;
      dk[j] = d;
      val[j] = c.value;
      if (q == SHARD_CAND - 1) s_tiekey[s] = ((unsigned)c.index & CAND_TIES) ? fkey(c.value) : 0u;
      best = d < best ? d : best;
    }
    if (tid == 0) {
      s_m = 0;
      s_bad = 0;
    }
    if (P.greedy) {  // largest value, then smallest index (sampling.cpp:73-76)
      best = block_reduce(best, MinU64{}, s_red);
      if (tid == 0) a.out_ids[row] = (int)(unsigned)(best & 0xffffffffull);
      __syncthreads();
      continue;
    }
    const int k = P.top_k;
    if (k < 1 || k > SHARD_CAND || k >= a.Vtot) {  // outside what 64 candidates per shard decide
      if (tid == 0) {
        atomicOr(a.errflags, C4S_DEVERR_SHARD);
        a.out_ids[row] = -1;
      }
      __syncthreads();
      continue;
    }
    __syncthreads();
    // rank of every candidate in descending (value) / ascending index order:
    // binary searches in the shards' sorted blocks
    int myr[NC / NT];
#pragma unroll
    for (int t = 0; t < NC / NT; ++t) {
      const int j = tid + t * NT;
      myr[t] = -1;
      if (j < n) {
        const unsigned long long K = dk[j];
        int r = 0;
        for (int s = 0; s < G; ++s) {
          const unsigned long long* blk = dk + s * SHARD_CAND;
          int lo = 0, hi = SHARD_CAND;
          while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (blk[mid] < K) lo = mid + 1;
            else hi = mid;
          }
          r += lo;
        }
        myr[t] = r;
        if (r == k - 1) s_tk = fkey(val[j]);  // top_k threshold: the k-th largest value
      }
    }
    csync();
    const unsigned tk = s_tk;
#pragma unroll
    for (int t = 0; t < NC / NT; ++t) {
      const int j = tid + t * NT;
      if (j < n && fkey(val[j]) >= tk) {
        sv[myr[t]] = j;
        atomicAdd(&s_m, 1);
      }
    }
    if (tid < G && s_tiekey[tid] != 0u && s_tiekey[tid] == tk) s_bad = 1;
    csync();
    if (s_bad) {
      if (tid == 0) {
        atomicOr(a.errflags, C4S_DEVERR_SHARD);
        a.out_ids[row] = -1;
      }
      __syncthreads();
      continue;
    }
    const int m = s_m;  // survivors of top_k: descending ranks [0, m)
    // ascending (value, index) order: the reverse, with equal values kept in index order
    const float maxv = val[sv[0]];
    for (int r = tid; r < m; r += NT) {
      const int j = sv[r];
      const unsigned f = fkey(val[j]);
      int r0 = r, r1 = r;
      while (r0 > 0 && fkey(val[sv[r0 - 1]]) == f) --r0;
      while (r1 < m - 1 && fkey(val[sv[r1 + 1]]) == f) ++r1;
      const int pos = (m - 1 - r1) + (r - r0);
      ord[pos] = j;
      pr[pos] = prob(val[j], maxv);
    }
    csync();
    // top_p (sampling.cpp:54-68): the sum and the running sum in ascending order
    if (tid == 0) {
      double sum = 0.0;
      for (int r = 0; r < m; ++r) sum += pr[r];
      s_sum = sum;
    }
    csync();
    const double sum = s_sum;
    for (int r = tid; r < m; r += NT) pr[r] = pr[r] / sum;
    csync();
    if (tid == 0) {
      const double thr = 1.0 - (double)P.top_p;
      double cum = 0.0;
      int nrem = 0;
      for (int r = 0; r < m; ++r) {
        cum += pr[r];
        if (cum <= thr) ++nrem;
        else break;
      }
      const int mk = P.min_tokens_to_keep;
      if (mk > 0) nrem = max(0, min(nrem, m - mk));
      s_keep = nrem;
    }
    csync();
    const int keep = s_keep;
    const int nk = m - keep;
    // the draw (text2semantic.cpp:150-165), in index order over the kept candidates
    const float mv = nk > 0 ? fmaxf(-1e30f, val[ord[m - 1]]) : -1e30f;
    for (int p = keep + tid; p < m; p += NT) {
      const int j = ord[p];
      const unsigned gi = (unsigned)(dk[j] & 0xffffffffull);
      int r = 0;
      for (int l = keep; l < m; ++l) r += (unsigned)(dk[ord[l]] & 0xffffffffull) < gi;
      sv[r] = j;
      pr[r] = prob(val[j], mv);
    }
    csync();
    if (tid == 0) {
      double s2 = 0.0;
      for (int r = 0; r < nk; ++r) s2 += pr[r];
      unsigned long long x = a.rng[row];
      x ^= x << 13;
      x ^= x >> 7;
      x ^= x << 17;
      a.rng[row] = x;
      const double rr = (double)(x >> 11) / 9007199254740992.0 * s2;
      int tok = a.Vtot - 1;
      if (nk == 0 || rr <= 0.0) {
        tok = 0;  // the reference's first index satisfies r <= acc
      } else {
        double acc = 0.0;
        for (int r = 0; r < nk; ++r) {
          acc += pr[r];
          if (rr <= acc) {
            tok = (int)(unsigned)(dk[sv[r]] & 0xffffffffull);
            break;
          }
        }
      }
      a.out_ids[row] = tok;
    }
    __syncthreads();
  }
}

}  // namespace c4s
