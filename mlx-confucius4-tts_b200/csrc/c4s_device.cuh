// c4s_device.cuh -- device building blocks for the T2S sampling kernels:
// order-preserving keys, block reductions/scans, shared-memory bitonic sort,
// bulk-async (TMA engine) row staging with a bounded mbarrier wait.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace c4s {

constexpr int NT = 256;               // threads per CTA (8 warps)
constexpr int NWARP = NT / 32;
constexpr int NBIN = 256;             // distance-from-max bins
constexpr float BIN_SCALE = 4.0f;     // bins are 1/4 logit wide, bin 255 = overflow
constexpr int LIST_CAP = 1024;        // candidates sorted in shared memory
constexpr int SEQ_MAX = 96;           // <= this many survivors: exact sequential sums
constexpr int MAX_VOCAB = 32768;      // row must fit in shared memory
constexpr unsigned FULL = 0xffffffffu;
constexpr unsigned long long KEY_MAX = ~0ull;

// CTA barrier of the NT threads (named barrier 1). It is the non-aligned
// form (barrier.sync, not bar.sync = barrier.sync.aligned): a warp may reach
// it with its lanes diverged (e.g. right after a branch only lane 0 takes,
// such as a bounded wait on an mbarrier), which the aligned form leaves
// undefined. Orders shared- and global-memory accesses among the participants.
__device__ __forceinline__ void csync() { asm volatile("barrier.sync 1, %0;" ::"n"(NT) : "memory"); }

// ---------------------------------------------------------------------------
// Keys. fkey() maps a float to a uint32 whose unsigned order is the float
// order, with -0 folded onto +0 so that key equality is float equality.
// ckey() appends the index: ascending ckey order is ascending (value, index),
// the canonical order of the top-p sort.
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned fkey(float f) {
  unsigned u = __float_as_uint(f);
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(unsigned k) {
  unsigned u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}
__device__ __forceinline__ unsigned long long ckey(float f, int i) {
  return ((unsigned long long)fkey(f) << 32) | (unsigned)i;
}
__device__ __forceinline__ int ckey_idx(unsigned long long k) { return (int)(unsigned)(k & 0xffffffffull); }

// Distance-from-max bin: non-increasing in y, so bins partition the ascending
// value order into contiguous ranges. -inf (and anything 64+ below the max)
// lands in the overflow bin NBIN-1.
__device__ __forceinline__ int vbin(float m, float y) {
  float t = __fmul_rn(__fsub_rn(m, y), BIN_SCALE);
  t = fminf(t, (float)(NBIN - 1));
  return (int)t;
}

// ---------------------------------------------------------------------------
// Warp / block reductions and scans (all threads of the CTA must call).
// `red` is shared scratch of at least NWARP elements of the value type.
// ---------------------------------------------------------------------------
template <typename T, typename Op>
__device__ __forceinline__ T warp_reduce(T v, Op op) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(FULL, v, o));
  return v;
}

template <typename T, typename Op>
__device__ __forceinline__ T block_reduce(T v, Op op, T* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_reduce(v, op);
  if (lane == 0) red[warp] = v;
  csync();
  T r = red[0];
#pragma unroll
  for (int w = 1; w < NWARP; ++w) r = op(r, red[w]);
  csync();
  return r;
}

struct MaxF { __device__ float operator()(float a, float b) const { return fmaxf(a, b); } };
struct SumU64 { __device__ unsigned long long operator()(unsigned long long a, unsigned long long b) const { return a + b; } };
struct MaxU64 { __device__ unsigned long long operator()(unsigned long long a, unsigned long long b) const { return a > b ? a : b; } };
struct MinU64 { __device__ unsigned long long operator()(unsigned long long a, unsigned long long b) const { return a < b ? a : b; } };
struct SumI { __device__ int operator()(int a, int b) const { return a + b; } };

// Exclusive scan of one uint64 per thread over the CTA; *total gets the sum.
__device__ __forceinline__ unsigned long long block_exscan_u64(unsigned long long v, unsigned long long* red,
                                                               unsigned long long* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    unsigned long long y = __shfl_up_sync(FULL, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) red[warp] = x;
  csync();
  unsigned long long wbase = 0, tot = 0;
#pragma unroll
  for (int w = 0; w < NWARP; ++w) {
    unsigned long long t = red[w];
    if (w < warp) wbase += t;
    tot += t;
  }
  csync();
  *total = tot;
  return wbase + x - v;
}

// Exclusive scan of one int per thread over the CTA.
__device__ __forceinline__ int block_exscan_i32(int v, int* red, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(FULL, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) red[warp] = x;
  csync();
  int wbase = 0, tot = 0;
#pragma unroll
  for (int w = 0; w < NWARP; ++w) {
    int t = red[w];
    if (w < warp) wbase += t;
    tot += t;
  }
  csync();
  *total = tot;
  return wbase + x - v;
}

// ---------------------------------------------------------------------------
// Warp 0 search over 256 bins in a given logical order: finds the first
// logical position c whose inclusive running sum exceeds (strict=true) or
// reaches (strict=false) `target`. get(j) returns the value of logical bin j.
// Results are written by lane 0 to *c_out (NBIN if none) and *before_out
// (sum of logical bins < c). Only warp 0 may call.
// ---------------------------------------------------------------------------
template <typename T, typename Get>
__device__ __forceinline__ void warp_find_bin(Get get, T target, bool strict, int* c_out, T* before_out) {
  const int lane = threadIdx.x & 31;
  T loc[8];
  T s = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) { loc[j] = get(lane * 8 + j); s += loc[j]; }
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
    if (lane == 0) { *c_out = NBIN; *before_out = tot; }
    return;
  }
  const int L = __ffs(bal) - 1;
  if (lane == L) {
    T run = incl - s;
    int c = L * 8 + 7;
    T before = run;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const bool h = strict ? (run + loc[j] > target) : (run + loc[j] >= target);
      if (h) { c = L * 8 + j; before = run; break; }
      run += loc[j];
    }
    *c_out = c;
    *before_out = before;
  }
}

// ---------------------------------------------------------------------------
// Bitonic sort (ascending) of n = power of two uint64 keys; `a` may be in
// shared or global memory (the CTA-wide barrier orders both).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void bitonic_sort_u64(unsigned long long* a, int n) {
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n; i += NT) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long x = a[i], y = a[ixj];
          const bool up = ((i & k) == 0);
          if ((x > y) == up) { a[i] = y; a[ixj] = x; }
        }
      }
      csync();
    }
  }
}

__device__ __forceinline__ int next_pow2(int n) {
  int p = 1;
  while (p < n) p <<= 1;
  return p;
}

// ---------------------------------------------------------------------------
// Bulk-async copy (TMA engine, non-tensor form) with an mbarrier. No cluster
// multicast is used anywhere in this library.
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned smem_u32(const void* p) {
  return (unsigned)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(unsigned long long* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(unsigned long long* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// Arrive once (release semantics at CTA scope).
__device__ __forceinline__ void mbar_arrive(unsigned long long* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, unsigned phase) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait (about 2 s of wall time); false if it gave up. Polls with a
// 128 ns back-off.
__device__ __forceinline__ bool mbar_wait_bounded(unsigned long long* bar, unsigned phase) {
  if (mbar_try_wait(bar, phase)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (unsigned it = 0; it < (1u << 30); ++it) {
    // back off between polls: a spinning warp takes issue slots from the
    // resident CTAs that have work
    __nanosleep(128);
    if (mbar_try_wait(bar, phase)) return true;
    if ((it & 15u) == 15u && globaltimer_ns() - t0 > 2000000000ull) return false;
  }
  return false;
}
// Programmatic dependent launch: a kernel launched with programmatic stream
// serialisation may start while the previous kernel of its stream finishes;
// grid_dep_wait() returns once that kernel has completed and its writes are
// visible (at once when there is none), grid_dep_launch() lets the next
// kernel start launching.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// 2^x by the hardware approximation (subnormal results flushed to zero).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

}  // namespace c4s

namespace c4s {

// ---------------------------------------------------------------------------
// Warp bitonic sort (ascending) of n <= 32*E uint64 keys held in `buf`
// (shared memory), by one full warp; blocked layout, lane l owns positions
// [l*E, l*E+E). Pads with KEY_MAX beyond n.
// ---------------------------------------------------------------------------
template <int E>
__device__ __forceinline__ void warp_sort_e(unsigned long long* buf, int n) {
  const int lane = threadIdx.x & 31;
  unsigned long long v[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int p = lane * E + e;
    v[e] = p < n ? buf[p] : KEY_MAX;
  }
#pragma unroll
  for (int k = 2; k <= 32 * E; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j < E) {
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const int e2 = e ^ j;
          if (e2 > e) {
            const bool up = ((lane * E + e) & k) == 0;
            const unsigned long long a = v[e], b = v[e2];
            if (up ? (a > b) : (a < b)) { v[e] = b; v[e2] = a; }
          }
        }
      } else {
        const int lj = j / E;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const int p = lane * E + e;
          const unsigned long long o = __shfl_xor_sync(FULL, v[e], lj);
          const bool keep_min = (((p & j) == 0) == ((p & k) == 0));
          v[e] = keep_min ? (o < v[e] ? o : v[e]) : (o > v[e] ? o : v[e]);
        }
      }
    }
  }
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int p = lane * E + e;
    if (p < n) buf[p] = v[e];
  }
  __syncwarp();
}

// n <= 128; whole warp must call.
__device__ __forceinline__ void warp_sort(unsigned long long* buf, int n) {
  if (n <= 1) { __syncwarp(); return; }
  if (n <= 32) warp_sort_e<1>(buf, n);
  else if (n <= 64) warp_sort_e<2>(buf, n);
  else warp_sort_e<4>(buf, n);
}

}  // namespace c4s

namespace c4s {

// Ampere-style asynchronous global->shared copies (per-thread groups).
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Bulk prefetch of [src, src + bytes) into L2 (src 16-byte aligned, bytes a
// multiple of 16); no completion to wait for.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

}  // namespace c4s
