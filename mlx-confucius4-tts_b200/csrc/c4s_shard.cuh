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

struct ShardArgs {
  const float* logits;   // this shard's columns: row r at logits + r * ld
  int B, Vs;             // rows, shard width
  long long ld;
  int voff, Vtot;        // global index of column 0, full vocabulary
  const int* hist;
  const long long* hist_off;
  long long hist_total;
  const c4s_row_params* params;
  int params_stride;
  const unsigned char* active;
  c4s_candidate* cand;   // [B][SHARD_CAND]
  unsigned* errflags;
};

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
// (~fkey(value) << 32 | local index): largest value first, ties by index.
__device__ __forceinline__ void shard_emit(const ShardArgs& a, int row, const float* srow,
                                           const unsigned long long* list, bool ties) {
  const int t = threadIdx.x;
  if (t < SHARD_CAND) {
    const unsigned long long k = list[t];
    const int li = (int)(unsigned)(k & 0xffffffffull);
    unsigned gi = (unsigned)(a.voff + li);
    if (t == SHARD_CAND - 1 && ties) gi |= CAND_TIES;
    c4s_candidate c;
    c.value = srow[li];
    c.index = (int)gi;
    a.cand[(long long)row * SHARD_CAND + t] = c;
  }
}

__global__ void __launch_bounds__(NT) shard_kernel(ShardArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned long long* list = reinterpret_cast<unsigned long long*>(smem);
  float* srow = reinterpret_cast<float*>(smem + (size_t)SHARD_LIST * 8);
  unsigned* bitmap = reinterpret_cast<unsigned*>(srow + align_up((size_t)a.Vs, 4));
  __shared__ unsigned s_wk[NWARP];
  __shared__ unsigned s_hist[256];
  __shared__ int s_cnt, s_digit, s_want;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int Vs = a.Vs;
  for (int row = blockIdx.x; row < a.B; row += gridDim.x) {
    if (a.active && !a.active[row]) continue;
    const c4s_row_params P = a.params[(long long)row * a.params_stride];
    const float* g = a.logits + (long long)row * a.ld;
    // 1. stage the shard's row (16-byte loads when the row is aligned)
    if ((((uintptr_t)g) & 15) == 0) {
      const float4* g4 = reinterpret_cast<const float4*>(g);
      float4* s4 = reinterpret_cast<float4*>(srow);
      for (int i = tid; i < Vs / 4; i += NT) s4[i] = __ldg(g4 + i);
      for (int i = (Vs & ~3) + tid; i < Vs; i += NT) srow[i] = __ldg(g + i);
    } else {
      for (int i = tid; i < Vs; i += NT) srow[i] = __ldg(g + i);
    }
    // 2. repetition penalty over the history ids inside this shard
    const bool pen = P.repetition_penalty != 1.0f && a.hist_off != nullptr;
    long long h0 = 0, h1 = 0;
    if (pen) {
      h0 = a.hist_off[row];
      h1 = a.hist_off[row + 1];
      if (h0 < 0 || h1 < h0 || h1 > a.hist_total) {
        if (tid == 0) atomicOr(a.errflags, C4S_DEVERR_HIST_RANGE);
        h0 = h1 = 0;
      }
      for (int i = tid; i < (Vs + 31) / 32; i += NT) bitmap[i] = 0u;
    }
    if (tid == 0) s_cnt = 0;
    __syncthreads();
    if (pen) {
      const float pv = P.repetition_penalty;
      const float rpv = __frcp_rn(pv);
      for (long long j = h0 + tid; j < h1; j += NT) {
        const int t = a.hist[j];
        const unsigned u = (unsigned)t - (unsigned)a.voff;
        if (t >= 0 && u < (unsigned)Vs) {
          const unsigned bit = 1u << (u & 31);
          const unsigned old = atomicOr(&bitmap[u >> 5], bit);
          if (!(old & bit)) {
            const float s = srow[u];
            srow[u] = (s < 0.0f) ? __fmul_rn(s, pv) : div_rn(s, pv, rpv);
          }
        }
      }
      __syncthreads();
    }
    // 3. temperature (sampled rows) and each thread's largest key
    const bool temper = !P.greedy && !(P.temperature == 1.0f || P.temperature <= 0.0f);
    const float T = P.temperature;
    const float rT = __frcp_rn(T);
    unsigned tmax = 0u;
    for (int i = tid; i < Vs; i += NT) {
      float v = srow[i];
      if (temper) {
        v = div_rn(v, T, rT);
        srow[i] = v;
      }
      tmax = max(tmax, fkey(v));
    }
    // 4. a lower bound on the 64th largest key: in every warp 8 lanes hold an
    //    element at least as large as the warp's 8th-largest lane maximum, so
    //    at least 64 elements are >= the least of the 8 warps' values.
    int rank = 0;
    for (int s = 0; s < 32; ++s) {
      const unsigned o = __shfl_sync(FULL, tmax, s);
      rank += (o > tmax) || (o == tmax && s < lane);
    }
    const unsigned sel = __ballot_sync(FULL, rank == 7);
    const unsigned wk = __shfl_sync(FULL, tmax, __ffs(sel) - 1);
    if (lane == 0) s_wk[warp] = wk;
    __syncthreads();
    unsigned tau0 = s_wk[0];
#pragma unroll
    for (int w = 1; w < NWARP; ++w) tau0 = min(tau0, s_wk[w]);
    // 5. every element >= the bound into the list (any order)
    for (int i0 = 0; i0 < Vs; i0 += NT) {
      const int i = i0 + tid;
      const unsigned k = i < Vs ? fkey(srow[i]) : 0u;
      const bool take = i < Vs && k >= tau0;
      const unsigned m = __ballot_sync(FULL, take);
      int base = 0;
      if (lane == 0 && m) base = atomicAdd(&s_cnt, __popc(m));
      base = __shfl_sync(FULL, base, 0);
      if (take) {
        const int pos = base + __popc(m & ((1u << lane) - 1u));
        if (pos < SHARD_LIST) list[pos] = ((unsigned long long)(~k) << 32) | (unsigned)i;
      }
    }
    __syncthreads();
    const int n0 = s_cnt;
    if (n0 >= SHARD_CAND && n0 <= SHARD_LIST) {
      const int n2 = next_pow2(n0);
      for (int i = n0 + tid; i < n2; i += NT) list[i] = KEY_MAX;
      __syncthreads();
      bitonic_sort_u64(list, n2);
      const bool ties = n0 > SHARD_CAND && (list[SHARD_CAND] >> 32) == (list[SHARD_CAND - 1] >> 32);
      shard_emit(a, row, srow, list, ties);
    } else {
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
      shard_emit(a, row, srow, list, eq_before > want);
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(NT) merge_kernel(MergeArgs a) {
  __shared__ unsigned long long key[SHARD_CAND * MAX_SHARDS];  // ascending (value, global index)
  __shared__ double pr[SHARD_CAND * MAX_SHARDS];
  __shared__ int ord[SHARD_CAND * MAX_SHARDS];
  __shared__ unsigned s_tiekey[MAX_SHARDS];
  __shared__ unsigned long long s_red[NWARP];
  __shared__ int s_first, s_keep, s_bad;
  const int tid = threadIdx.x;
  const int n = a.G * SHARD_CAND;
  const int n2 = next_pow2(n);
  for (int row = blockIdx.x; row < a.B; row += gridDim.x) {
    if (a.active && !a.active[row]) {
      if (tid == 0) a.out_ids[row] = -1;
      continue;
    }
    const c4s_row_params P = a.params[(long long)row * a.params_stride];
    unsigned long long best = 0ull;
    for (int j = tid; j < n2; j += NT) {
      unsigned long long k = 0ull;  // padding sorts first
      if (j < n) {
        const int s = j / SHARD_CAND, q = j % SHARD_CAND;
        const c4s_candidate c = a.cand[(long long)s * a.shard_stride + (long long)row * SHARD_CAND + q];
        const unsigned gi = (unsigned)c.index & ~CAND_TIES;
        k = ckey(c.value, (int)gi);
        if (q == SHARD_CAND - 1) s_tiekey[s] = ((unsigned)c.index & CAND_TIES) ? fkey(c.value) : 0u;
        // greedy: largest value, then smallest index
        const unsigned long long gk = ((unsigned long long)fkey(c.value) << 32) | (0xffffffffu - gi);
        best = gk > best ? gk : best;
      }
      key[j] = k;
    }
    if (P.greedy) {
      best = block_reduce(best, MaxU64{}, s_red);
      if (tid == 0) a.out_ids[row] = (int)(0xffffffffu - (unsigned)(best & 0xffffffffull));
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
    bitonic_sort_u64(key, n2);
    // top_k: threshold = k-th largest; survivors = every candidate >= it
    const unsigned tk = (unsigned)(key[n2 - k] >> 32);
    if (tid == 0) s_bad = 0;
    for (int j = n2 - n + tid; j <= n2 - k; j += NT) {
      if ((unsigned)(key[j] >> 32) >= tk && (j == n2 - n || (unsigned)(key[j - 1] >> 32) < tk)) s_first = j;
    }
    csync();
    if (tid < a.G && s_tiekey[tid] != 0u && s_tiekey[tid] == tk) s_bad = 1;
    csync();
    if (s_bad) {
      if (tid == 0) {
        atomicOr(a.errflags, C4S_DEVERR_SHARD);
        a.out_ids[row] = -1;
      }
      __syncthreads();
      continue;
    }
    const int first = s_first;
    // top_p over the survivors in ascending (value, index) order
    const float maxv = fkey_inv((unsigned)(key[n2 - 1] >> 32));
    for (int j = first + tid; j < n2; j += NT) pr[j] = prob(fkey_inv((unsigned)(key[j] >> 32)), maxv);
    csync();
    if (tid == 0) {
      double sum = 0.0;
      for (int j = first; j < n2; ++j) sum += pr[j];
      const double thr = 1.0 - (double)P.top_p;
      double cum = 0.0;
      int nrem = 0;
      for (int j = first; j < n2; ++j) {
        cum += pr[j] / sum;
        if (cum <= thr) ++nrem;
        else break;
      }
      int keep = first + nrem;
      const int mk = P.min_tokens_to_keep;
      if (mk > 0) keep = max(first, min(keep, n2 - mk));
      s_keep = keep;
    }
    csync();
    const int keep = s_keep;
    const int nk = n2 - keep;
    // the draw, in index order over the kept candidates
    const float mv = fmaxf(-1e30f, fkey_inv((unsigned)(key[n2 - 1] >> 32)));
    for (int j = keep + tid; j < n2; j += NT) {
      const unsigned gi = (unsigned)(key[j] & 0xffffffffull);
      int r = 0;
      for (int l = keep; l < n2; ++l) r += (unsigned)(key[l] & 0xffffffffull) < gi;
      ord[r] = j;
      pr[j] = prob(fkey_inv((unsigned)(key[j] >> 32)), mv);
    }
    csync();
    if (tid == 0) {
      double sum = 0.0;
      for (int r = 0; r < nk; ++r) sum += pr[ord[r]];
      unsigned long long x = a.rng[row];
      x ^= x << 13;
      x ^= x >> 7;
      x ^= x << 17;
      a.rng[row] = x;
      const double rr = (double)(x >> 11) / 9007199254740992.0 * sum;
      int tok = a.Vtot - 1;
      if (nk == 0 || rr <= 0.0) {
        tok = 0;  // the reference's first index satisfies r <= acc
      } else {
        double acc = 0.0;
        for (int r = 0; r < nk; ++r) {
          const int j = ord[r];
          acc += pr[j];
          if (rr <= acc) {
            tok = (int)(unsigned)(key[j] & 0xffffffffull);
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
