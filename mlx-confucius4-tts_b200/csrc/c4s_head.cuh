// c4s_head.cuh -- the T2S LM head on sm_100a tensor cores (tcgen05 / TMEM).
//
// The reference computes, per decode step (text2semantic.cpp:118-121 single
// stream, :283-286 batched; nn.cpp:11-16 linear, nn.cpp:73-83 layer_norm):
//
//     y      = layer_norm(h; final_norm.weight, final_norm.bias)   (biased variance)
//     logits = y W^T + b,  W = semantic_head.weight (N x d, out x in)
//
// and hands the logits row to the sampling stage. Here both stay on the
// device: ln_kernel writes y in bf16 (the GEMM operand type), and
// head_gemm_kernel computes logits = y W^T + b with fp32 accumulation:
//
//   one CTA per 128 x 128 tile of the [B, N] output, 18 warps --
//     warp 0 (one lane)  TMA producer: 128 x 64 bf16 tiles of y and W per
//                        k-block by cp.async.bulk.tensor (128-byte swizzle)
//                        into a 6-stage shared-memory ring (full/empty
//                        mbarriers);
//     warp 1             allocates 128 TMEM columns; one lane issues
//                        tcgen05.mma kind::f16 (M 128, N 128, K 16; bf16 in,
//                        fp32 accumulator in TMEM), tcgen05.commit frees each
//                        stage and finally signals the accumulator;
//     warps 2-17         epilogue, four per TMEM lane quarter: tcgen05.ld of
//                        a 32-column chunk of their 32 TMEM lanes (rows),
//                        + bias, fp32 stores of the logits.
//   No cluster, no multicast: every TMA load reads this GPU's own memory.
//   Every mbarrier wait is bounded (about 1 s); a wait that gives up sets
//   C4S_DEVERR_TIMEOUT, the roles stop, the MMAs issued so far are committed
//   and waited for, and the TMEM is freed before the CTA exits.
//
// c4s_head_sample then runs the sampling step (c4s_sample) on the logits,
// with programmatic dependent launch between the three kernels.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

namespace c4s {

constexpr int HG_BM = 128, HG_BN = 128, HG_BK = 64, HG_ST = 6;
constexpr int HG_EPI_WARPS = 16;                   // four per TMEM lane quarter, each a quarter of the columns
constexpr int HG_THREADS = 64 + 32 * HG_EPI_WARPS;  // producer warp, MMA warp, epilogue warps
constexpr unsigned HG_TILE_BYTES = (unsigned)HG_BM * HG_BK * 2;          // one 128 x 64 bf16 tile: 16 KB
constexpr unsigned HG_STAGE_BYTES = 2 * HG_TILE_BYTES;                    // y tile + W tile
constexpr size_t HG_SMEM = (size_t)HG_ST * HG_STAGE_BYTES + 1024;        // + alignment slack (1024-byte tiles)
// the epilogue's transposed chunks (all warps' 32 x 33-float chunks) reuse the pipeline buffers
static_assert(HG_EPI_WARPS % 4 == 0 && (HG_BN / 32) % (HG_EPI_WARPS / 4) == 0, "whole chunks per epilogue warp");
static_assert(4 * (HG_BN / 32) * 32 * 33 * 4 <= HG_ST * HG_STAGE_BYTES, "epilogue buffers fit the pipeline's");
constexpr unsigned HG_TMEM_COLS = 128;                                   // fp32 accumulator, 128 lanes x 128 columns
// Instruction descriptor of tcgen05.mma kind::f16: D fp32 (bits 4-5 = 1),
// A and B bf16 (bits 7-9 = 1, 10-12 = 1), both K-major (bits 15, 16 = 0),
// N >> 3 at bits 17-22, M >> 4 at bits 24-28.
constexpr unsigned HG_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((unsigned)(HG_BN >> 3) << 17) |
                              ((unsigned)(HG_BM >> 4) << 24);

struct HeadGemmArgs {
  float* logits;
  long long ldl;
  const float* bias;
  int M, N, K;
  unsigned* errflags;
};

// ---- tcgen05 / TMA primitives (inline PTX) ----------------------------------
__device__ __forceinline__ void tmem_alloc(unsigned* dst, unsigned ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(unsigned taddr, unsigned ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void umma_bf16(unsigned tmem_d, unsigned long long adesc, unsigned long long bdesc,
                                          unsigned accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(HG_IDESC), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(unsigned long long* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<unsigned long long>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
// Shared-memory matrix descriptor of a K-major 128-byte-swizzled tile (rows of
// 64 bf16 = 128 B, 8-row swizzle atoms of 1024 B): start address >> 4 (bits
// 0-13), leading byte offset 16 B (unused by swizzled K-major layouts; field
// 1), stride byte offset 1024 B between 8-row groups (bits 32-45), version 1
// (bits 46-47), layout SWIZZLE_128B (2 at bits 61-63). The tile must be
// 1024-byte aligned; the K = 16 steps inside the 64-wide tile advance the
// start address by 32 B.
__device__ __forceinline__ unsigned long long sw128_desc(const void* tile) {
  const unsigned a = smem_u32(tile);
  return (unsigned long long)((a & 0x3FFFFu) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// 32 TMEM lanes x 32 consecutive 32-bit columns into 32 registers per thread
// (thread t of the warp gets lane base + t).
__device__ __forceinline__ void tmem_ld32(unsigned taddr, unsigned (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Bounded wait for an mbarrier phase (about 1 s of wall time).
__device__ __forceinline__ bool mbar_wait_1s(unsigned long long* bar, unsigned parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (unsigned it = 0; it < (1u << 30); ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 63u && globaltimer_ns() - t0 > 1000000000ull) return false;
  }
  return false;
}

// ---- LayerNorm (nn.cpp:73-83) -----------------------------------------------
// One warp per row: mean, biased variance (two passes over the row in
// registers, fp32), y = (x - mean) / sqrt(var + eps) * gamma + beta rounded
// to bf16. d is a multiple of 64, at most HN_MAXD.
constexpr int HN_MAXD = 8192;
constexpr int HN_WARPS = 8;
__global__ void __launch_bounds__(32 * HN_WARPS) ln_kernel(const unsigned short* __restrict__ h, long long ldh,
                                                           int B, int d, const float* __restrict__ gamma,
                                                           const float* __restrict__ beta, float eps,
                                                           unsigned short* __restrict__ y) {
  grid_dep_wait();                                 // y may still be read by the previous step's GEMM
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * HN_WARPS + (threadIdx.x >> 5);
  if (row >= B) return;
  const unsigned short* hr = h + (long long)row * ldh;
  constexpr int MAXV = HN_MAXD / 256;              // 8-byte vectors (4 bf16) per lane
  float x[MAXV * 4];
  const int nv = d / 128;                          // vectors of 4 per lane
  float s = 0.0f;
#pragma unroll
  for (int v = 0; v < MAXV; ++v) {
    if (v < nv) {
      const uint2 w = reinterpret_cast<const uint2*>(hr)[v * 32 + lane];
      x[4 * v + 0] = __uint_as_float(w.x << 16);
      x[4 * v + 1] = __uint_as_float(w.x & 0xffff0000u);
      x[4 * v + 2] = __uint_as_float(w.y << 16);
      x[4 * v + 3] = __uint_as_float(w.y & 0xffff0000u);
      s += (x[4 * v] + x[4 * v + 1]) + (x[4 * v + 2] + x[4 * v + 3]);
    }
  }
  s = warp_reduce(s, [](float a, float b) { return a + b; });
  const float mean = s / (float)d;
  float q = 0.0f;
#pragma unroll
  for (int v = 0; v < MAXV; ++v)
    if (v < nv)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float t = x[4 * v + c] - mean;
        q = fmaf(t, t, q);
      }
  q = warp_reduce(q, [](float a, float b) { return a + b; });
  const float sd = sqrtf(q / (float)d + eps);
  unsigned short* yr = y + (long long)row * d;
#pragma unroll
  for (int v = 0; v < MAXV; ++v) {
    if (v < nv) {
      unsigned o[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int col = 4 * (v * 32 + lane) + c;
        const float g = gamma ? gamma[col] : 1.0f, bb = beta ? beta[col] : 0.0f;
        const float t = fmaf((x[4 * v + c] - mean) / sd, g, bb);
        // round to nearest even bf16 (finite inputs; NaN kept quiet)
        const unsigned u = __float_as_uint(t);
        o[c] = (u & 0x7fffffffu) > 0x7f800000u ? ((u >> 16) | 0x40u) : ((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
      }
      reinterpret_cast<uint2*>(yr)[v * 32 + lane] = make_uint2(o[0] | (o[1] << 16), o[2] | (o[3] << 16));
    }
  }
}

#ifdef C4S_TRACE
__device__ long long g_htrace[1024 * 8];
#define C4S_HTR(ph) (g_htrace[((blockIdx.y * gridDim.x + blockIdx.x) & 1023) * 8 + (ph)] = clock64())
#else
#define C4S_HTR(ph)
#endif

// ---- logits = y W^T + b on tcgen05 ------------------------------------------
__global__ void __launch_bounds__(HG_THREADS, 1) head_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                                                                  const __grid_constant__ CUtensorMap tmB,
                                                                  HeadGemmArgs g) {
  extern __shared__ unsigned char hsm_raw[];
  unsigned char* hsm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<unsigned long long>(hsm_raw) + 1023ull) & ~1023ull);
  __shared__ unsigned long long full[HG_ST], empty[HG_ST], accum;
  __shared__ unsigned tmem_base;
  __shared__ volatile int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * HG_BN, m0 = blockIdx.y * HG_BM;
  const int KB = g.K / HG_BK;
  const int kstart = KB > 0 ? (int)(blockIdx.x % (unsigned)KB) : 0;
  if (threadIdx.x == 0) C4S_HTR(0);
  if (threadIdx.x == 0) {
    for (int s = 0; s < HG_ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&accum, 1);
    abort_flag = 0;
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base, HG_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const unsigned tmem = tmem_base;
  grid_dep_wait();                                 // y is written by the LayerNorm kernel
  grid_dep_launch();
  if (threadIdx.x == 0) C4S_HTR(1);
  auto give_up = [&]() {
    atomicOr(g.errflags, C4S_DEVERR_TIMEOUT);
    abort_flag = 1;
  };
  if (warp == 0) {
    if (lane == 0) {
      // TMA producer. Every CTA of a row block reads the same activations:
      // each starts at its own k-block (and wraps around), so that the CTAs
      // running at once read different parts of them instead of queueing on
      // the same L2 lines; the CTAs of one weight tile start together, and
      // the second of them finds the tile in L2.
      for (int it = 0; it < KB && !abort_flag; ++it) {
        const int s = it % HG_ST;
        const unsigned ph = (unsigned)(it / HG_ST) & 1u;
        const int kb = (it + kstart) % KB;
        if (!mbar_wait_1s(&empty[s], ph ^ 1u)) { give_up(); break; }
        unsigned char* sa = hsm + (size_t)s * HG_STAGE_BYTES;
        mbar_arrive_expect_tx(&full[s], HG_STAGE_BYTES);
        tma_load_2d(sa, &tmA, kb * HG_BK, m0, &full[s]);
        tma_load_2d(sa + HG_TILE_BYTES, &tmB, kb * HG_BK, n0, &full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // MMA issuer: 4 MMAs of K = 16 per 64-wide k-block
      for (int it = 0; it < KB && !abort_flag; ++it) {
        const int s = it % HG_ST;
        const unsigned ph = (unsigned)(it / HG_ST) & 1u;
        if (!mbar_wait_1s(&full[s], ph)) { give_up(); break; }
        if (it == 0) C4S_HTR(2);
        if (it == KB / 2) C4S_HTR(3);
        tc_fence_after();
        const unsigned char* sa = hsm + (size_t)s * HG_STAGE_BYTES;
        const unsigned long long ad = sw128_desc(sa), bd = sw128_desc(sa + HG_TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < HG_BK / 16; ++kk)
          umma_bf16(tmem, ad + 2ull * kk, bd + 2ull * kk, (it | kk) != 0 ? 1u : 0u);
        umma_commit(&empty[s]);                     // the stage is free once these MMAs have read it
      }
      C4S_HTR(4);
      umma_commit(&accum);                          // every MMA issued so far has completed
    }
  } else {
    // epilogue warps: warp w reads TMEM lanes 32 (w % 4) .. + 31 = rows of the tile
    const bool ok = mbar_wait_1s(&accum, 0u);
    if (!ok) give_up();
    if (threadIdx.x == 64) C4S_HTR(5);
    tc_fence_after();
    if (ok && !abort_flag && KB > 0) {
      // warp w reads TMEM lane quarter q = w % 4 (the hardware's rule) and,
      // with the other warp of its quarter, half of the tile's columns. Each
      // 32 x 32 chunk (lane = row) goes through shared memory (the idle
      // pipeline buffers: every MMA, hence every load, has completed)
      // transposed, so that each store writes 32 consecutive logits of one
      // row; the warp's chunks are read from TMEM at once and transposed
      // before any store, so the loads' latency and the stores overlap.
      constexpr int NCH = HG_BN / 32 / (HG_EPI_WARPS / 4);   // chunks per warp
      const int q = warp & 3;
      const int c0 = ((warp - 2) >> 2) * NCH;                // the warp's first chunk
      float* T = reinterpret_cast<float*>(hsm) + (warp - 2) * (NCH * 32 * 33);
      const int rows = min(32, g.M - (m0 + 32 * q));   // rows of this warp's quarter inside the output
      float* obase = g.logits + (long long)(m0 + 32 * q) * g.ldl + n0 + lane;
      float bn[NCH];
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const int n = n0 + 32 * (c0 + c) + lane;
        bn[c] = (g.bias && n < g.N) ? __ldg(g.bias + n) : 0.0f;
      }
      {
        unsigned r[NCH][32];
#pragma unroll
        for (int c = 0; c < NCH; ++c)
          tmem_ld32(tmem + ((unsigned)(32 * q) << 16) + (unsigned)(32 * (c0 + c)), r[c]);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < NCH; ++c)
#pragma unroll
          for (int j = 0; j < 32; ++j) T[c * 32 * 33 + lane * 33 + j] = __uint_as_float(r[c][j]);   // bank (lane + j)
      }
      __syncwarp();
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        if (n0 + 32 * (c0 + c) + lane < g.N) {
          float* o = obase + 32 * (c0 + c);
          const float* t = T + c * 32 * 33 + lane;
#pragma unroll 8
          for (int rr = 0; rr < rows; ++rr) o[(long long)rr * g.ldl] = t[rr * 33] + bn[c];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) C4S_HTR(6);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, HG_TMEM_COLS);
  }
}

}  // namespace c4s
