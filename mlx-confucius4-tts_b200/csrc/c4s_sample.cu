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
#include <mutex>
#include <vector>
#include <string>

#include "../../include/c4s_sampling.h"
#include "c4s_device.cuh"
#include "c4s_general.cuh"
#include "c4s_fast.cuh"
#include "c4s_row.cuh"
#include "c4s_shard.cuh"
#include "c4s_fused.cuh"
#include "c4s_head.cuh"
#include "c4s_decode.cuh"
#include "c4s_qgemv.cuh"

namespace c4s {

// General kernel: every mode, rows up to MAX_VOCAB, row staged in shared memory.
__global__ void __launch_bounds__(NT, 4) rows_kernel(Args a) {
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
  for (int row = blockIdx.x; row < a.B; row += gridDim.x) {
    if (a.mode == MODE_SAMPLE && a.active && !a.active[row]) {
      if (threadIdx.x == 0) a.out_ids[row] = -1;
      continue;
    }
    if (!general_row(sa, row, rowbuf, bitmap, cnt, mass, lkey, pv, S, phase)) {
      // a bounded wait gave up (C4S_DEVERR_TIMEOUT): this CTA's remaining
      // rows are marked as not sampled instead of keeping stale ids
      if (a.mode != MODE_PROCESS && threadIdx.x == 0)
        for (int r = row; r < a.B; r += gridDim.x) a.out_ids[r] = -1;
      return;
    }
  }
}

// div_rn over n dividends and one divisor (test hook of the exact division).
__global__ void div_test_kernel(const float* x, float d, float* out, long long n) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = div_rn(x[i], d, __frcp_rn(d));
}

// Scratch of c4s_sample_static(), at file scope so that the entry point
// allocates nothing: STATIC_CTAS slabs of the general path's exact top-p sort
// (up to STATIC_MAX_VOCAB keys each, 2 MiB in all), and the error-flag word and
// path counters that the kernel writes.
constexpr int STATIC_CTAS = 16;
constexpr int STATIC_MAX_VOCAB = 16384;
static __device__ __align__(256) unsigned long long g_static_scratch[(size_t)STATIC_CTAS * STATIC_MAX_VOCAB];
static __device__ __align__(256) unsigned long long g_static_status[1 + C4S_NUM_COUNTERS];

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
  int chunk = 0;                               // rows per split-path launch sequence (<= K_CHUNK)
  unsigned long long* d_scratch = nullptr;
  unsigned* d_err = nullptr;
  unsigned long long* d_counters = nullptr;
  c4s_row_params* d_default_params = nullptr;  // one zeroed struct (argmax reads no field)
  int row_occ = 0;                             // resident row-kernel CTAs per SM
  int list_occ = 0;                            // resident list-kernel CTAs per SM
  int fused_occ = 0;                           // resident fused-kernel CTAs per SM
  int fused_small_occ = 0;                     //   and of its small-batch form
  int fused_mid_occ = 0;                       //   and of its two-per-SM form
  bool split_dirty = false;                    // a split-path launch sequence stopped early: its
                                               // queue counters may be stale until cleared
  c4s::RowJob* d_jobs = nullptr;               // fast path: per-row jobs of one chunk
  unsigned long long* d_lkeys = nullptr;       //   candidate lists [chunk][LCAP]
  unsigned long long* d_lsb = nullptr;
  int* d_defer_rows = nullptr;                 //   rows handed to the general path, then long lists
  int* d_order = nullptr;                      //   the row kernel's rows by cost class
  unsigned* d_defer_cnt = nullptr;
  int debug = 0;
  bool timing = false;                         // c4s_kernel_timing: events between fast-path launches
  std::vector<cudaEvent_t> tev;                //   TEV per recorded chunk: before the first kernel, then after
                                               //   the order, row, list, general and fused kernels
  std::vector<unsigned char> tev_mask;         //   per recorded chunk: bit k = kernel k ran
  size_t tev_used = 0;
  int cached_V = -1;
  int cached_occ = 0;
  size_t qg_smem_set = 0;                      // dynamic shared memory allowed for the quantized GEMV
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

// Timing events of the next recorded chunk (nullptr if they cannot be made):
// ev[0] before its first kernel, ev[k + 1] after kernel k (order, row, list,
// general, fused), recorded at once for kernels that do not run.
constexpr int TEV = 1 + C4S_NUM_KERNEL_TIMERS;
cudaEvent_t* timing_slot(c4s_ctx* ctx) {
  if (ctx->tev_used + TEV > ctx->tev.size()) {
    for (int i = 0; i < TEV; ++i) {
      cudaEvent_t e;
      if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
      ctx->tev.push_back(e);
    }
  }
  cudaEvent_t* ev = ctx->tev.data() + ctx->tev_used;
  ctx->tev_used += TEV;
  ctx->tev_mask.resize(ctx->tev_used / TEV);
  ctx->tev_mask.back() = 0;
  return ev;
}

// The fast path's kernels are launched with programmatic stream serialisation:
// each starts launching while its predecessor in the stream drains and waits
// in grid_dep_wait() before it reads what earlier launches wrote, so the gaps
// between the kernels of a step (and between steps) close.
template <typename K>
cudaError_t launch_pdl(K kern, int grid, int block, size_t smem, cudaStream_t st, const c4s::Args& a) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

int launch_rows(c4s_ctx* ctx, c4s::Args& a, void* stream) {
  using namespace c4s;
  if (a.B == 0) return C4S_OK;
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, C4S_ERR_CUDA, "cannot select the context's device");
  a.scratch = ctx->d_scratch;
  a.scratch_stride = ctx->scratch_stride;
  a.errflags = ctx->d_err;
  a.counters = ctx->d_counters;
  a.debug = ctx->debug;
  int lg = 0;
  while ((1 << lg) < a.V) ++lg;
  a.qscale = std::ldexp(1.0, 62 - std::max(lg, 1));
  cudaError_t e;
  const cudaStream_t st0 = (cudaStream_t)stream;
  const bool fused = a.B <= FUSED_MAX_ROWS ? !(ctx->debug & C4S_DEBUG_SPLIT_PATH) : (ctx->debug & C4S_DEBUG_FUSED_PATH) != 0;
  if (a.mode == MODE_SAMPLE && a.V <= F_MAXV && fused) {
    // fused path (small batches, or C4S_DEBUG_FUSED_PATH): one launch, every
    // row finished in its CTA; up to one row per SM the small-batch form
    a.defer_cnt = ctx->d_defer_cnt + FUSED_CNT;
    const size_t smem = fused_smem_bytes(a.V);
    if (ctx->fused_occ == 0) {
      int occ = 0, occ1 = 0, occ2 = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fused_kernel, NT, fused_smem_bytes(F_MAXV)) !=
              cudaSuccess || occ < 1 ||
          cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ1, fused_small_kernel, NT, fused_smem_bytes(F_MAXV)) !=
              cudaSuccess || occ1 < 1 ||
          cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ2, fused_mid_kernel, NT, fused_smem_bytes(F_MAXV)) !=
              cudaSuccess || occ2 < 1)
        return fail(ctx, C4S_ERR_CUDA, "fused kernel occupancy");
      ctx->fused_occ = occ;
      ctx->fused_small_occ = occ1;
      ctx->fused_mid_occ = occ2;
    }
    // one row per CTA while the rows fit the small form's (then the mid form's) CTAs
    const bool small = a.B <= (long long)ctx->fused_small_occ * ctx->num_sms;
    const bool mid = !small && a.B <= (long long)ctx->fused_mid_occ * ctx->num_sms;
    // every CTA uses two scratch slabs (blockIdx.x and grid + blockIdx.x)
    const int occ = small ? ctx->fused_small_occ : mid ? ctx->fused_mid_occ : ctx->fused_occ;
    const int grid = (int)std::min<long long>(std::min<long long>(a.B, (long long)occ * ctx->num_sms),
                                              (long long)ctx->scratch_ctas / 2);
    cudaEvent_t* ev = ctx->timing ? timing_slot(ctx) : nullptr;
    if (ev)
      for (int k = 0; k < TEV - 1; ++k) cudaEventRecord(ev[k], st0);
    e = small ? launch_pdl(fused_small_kernel, grid, NT, smem, st0, a)
        : mid ? launch_pdl(fused_mid_kernel, grid, NT, smem, st0, a)
              : launch_pdl(fused_kernel, grid, NT, smem, st0, a);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "fused kernel launch");
    if (ev) {
      cudaEventRecord(ev[TEV - 1], st0);
      ctx->tev_mask.back() = 1u << 4;
    }
    return C4S_OK;
  }
  if (a.mode == MODE_SAMPLE && a.V <= F_MAXV) {
    // split path (large batches, or C4S_DEBUG_SPLIT_PATH), per chunk of
    // ctx->chunk rows: row kernel -> list kernel -> general path for handed-back rows (->
    // masking of processed logits). Many list jobs run concurrently, one per
    // warp, which hides their latency at large batch sizes.
    a.jobs = ctx->d_jobs;
    a.lkeys = ctx->d_lkeys;
    a.lsb = ctx->d_lsb;
    a.defer_rows = ctx->d_defer_rows;
    a.big_rows = ctx->d_defer_rows + ctx->chunk;     // LIST_CLASSES queues of chunk rows
    a.chunk = ctx->chunk;
    a.defer_cnt = ctx->d_defer_cnt;
    if (ctx->row_occ == 0) {
      int occ = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, row_kernel, RT, R_SMEM) != cudaSuccess || occ < 1)
        return fail(ctx, C4S_ERR_CUDA, "row kernel occupancy");
      ctx->row_occ = occ;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, list_kernel, 32 * LIST_WARPS, LIST_SMEM) != cudaSuccess ||
          occ < 1)
        return fail(ctx, C4S_ERR_CUDA, "list kernel occupancy");
      ctx->list_occ = occ;
    }
    const cudaStream_t st = (cudaStream_t)stream;
    const size_t gsm = layout_for(a.V).total;
    if (ctx->split_dirty) {
      // an earlier sequence stopped after its row kernel: clear its queue counters
      e = cudaMemsetAsync(ctx->d_defer_cnt, 0, FUSED_CNT * sizeof(unsigned), st);
      if (e != cudaSuccess) return cuda_fail(ctx, e, "clear queue counters");
      ctx->split_dirty = false;
    }
    for (int c0 = 0; c0 < a.B; c0 += ctx->chunk) {
      Args ac = a;
      ac.B = std::min(ctx->chunk, a.B - c0);
      ac.logits = a.logits + (long long)c0 * a.ld;
      ac.params = a.params + (long long)c0 * a.params_stride;
      ac.rng = a.rng + c0;
      if (a.active) ac.active = a.active + c0;
      ac.out_ids = a.out_ids + c0;
      if (a.out_logits) ac.out_logits = a.out_logits + (long long)c0 * a.out_ld;
      if (a.hist_off) ac.hist_off = a.hist_off + c0;
      if (a.hist_len) ac.hist_len = a.hist_len + c0;
      const int g1 = (int)std::min<long long>(ac.B, (long long)ctx->row_occ * ctx->num_sms);
      cudaEvent_t* ev = ctx->timing ? timing_slot(ctx) : nullptr;
      if (ev) cudaEventRecord(ev[0], st);
      // more rows than CTAs, of varying kinds: the dearest rows go first
      ac.order = nullptr;
      if (ac.B > g1 && ac.params_stride != 0) {
        ac.order = ctx->d_order;
        e = launch_pdl(order_kernel, (ac.B + ORDER_NT - 1) / ORDER_NT, ORDER_NT, 0, st, ac);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "order kernel launch");
        if (ev) ctx->tev_mask.back() |= 1u;
      }
      if (ev) cudaEventRecord(ev[1], st);
      e = launch_pdl(row_kernel, g1, RT, R_SMEM, st, ac);
      if (e != cudaSuccess) return cuda_fail(ctx, e, "row kernel launch");
      // from here on the row kernel has taken queue tickets: a sequence that
      // stops before the general kernel (which clears them) leaves them stale
      ctx->split_dirty = true;
      if (ev) cudaEventRecord(ev[2], st);
      const int g2 = (int)std::min<long long>((ac.B + LIST_WARPS - 1) / LIST_WARPS,
                                                   (long long)ctx->list_occ * ctx->num_sms);
      e = (ctx->debug & C4S_DEBUG_FAIL_AFTER_ROW) ? cudaErrorInvalidConfiguration
                                                  : launch_pdl(list_kernel, g2, 32 * LIST_WARPS, LIST_SMEM, st, ac);
      if (e != cudaSuccess) return cuda_fail(ctx, e, "list kernel launch");
      if (ev) cudaEventRecord(ev[3], st);
      const int g3 = std::min(std::min(ac.B, ctx->num_sms), ctx->scratch_ctas);
      e = launch_pdl(defer_kernel, g3, NT, gsm, st, ac);
      if (e != cudaSuccess) return cuda_fail(ctx, e, "general kernel launch");
      ctx->split_dirty = false;
      if (ev) {
        cudaEventRecord(ev[4], st);
        cudaEventRecord(ev[5], st);
        ctx->tev_mask.back() |= 2u | 4u | 8u;
      }
      if (a.out_logits) mask_kernel<<<ac.B, NT, 0, st>>>(ac);
      e = cudaGetLastError();
      if (e != cudaSuccess) return cuda_fail(ctx, e, "fast path launch");
    }
    return C4S_OK;
  }
  const size_t smem = layout_for(a.V).total;
  const int occ = occupancy(ctx, a.V, smem);
  // one scratch slab per CTA: a context sized for few rows runs more rows per CTA
  const int grid = (int)std::min<long long>(std::min<long long>((long long)a.B, (long long)std::min(occ, 8) * ctx->num_sms),
                                            (long long)ctx->scratch_ctas);
  rows_kernel<<<grid, NT, smem, (cudaStream_t)stream>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(ctx, e, "rows_kernel launch");
  return C4S_OK;
}

void free_all(c4s_ctx* ctx) {
  for (cudaEvent_t e : ctx->tev) cudaEventDestroy(e);
  ctx->tev.clear();
  ctx->tev_used = 0;
  cudaFree(ctx->d_scratch);
  cudaFree(ctx->d_err);
  cudaFree(ctx->d_counters);
  cudaFree(ctx->d_default_params);
  cudaFree(ctx->d_jobs);
  cudaFree(ctx->d_lkeys);
  cudaFree(ctx->d_lsb);
  cudaFree(ctx->d_defer_rows);
  cudaFree(ctx->d_order);
  cudaFree(ctx->d_defer_cnt);
}

int check_common(c4s_ctx* ctx, int B, int V, long long ld) {
  if (!ctx) return C4S_ERR_INVALID;
  if (B < 0) return fail(ctx, C4S_ERR_INVALID, "B < 0");
  if (V < 1) return fail(ctx, C4S_ERR_INVALID, "V < 1");
  if (V > ctx->max_vocab) return fail(ctx, C4S_ERR_CAPACITY, "V above the context's max_vocab");
  if (ld < V) return fail(ctx, C4S_ERR_INVALID, "ld < V");
  return C4S_OK;
}

// Shard kernel launch: persistent CTAs over (row, shard) items.
int launch_shard(c4s_ctx* ctx, c4s::ShardArgs& a, void* stream) {
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, C4S_ERR_CUDA, "cannot select the context's device");
  const size_t smem = c4s::shard_smem_bytes(a.Vs);
  int occ = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, c4s::shard_kernel, c4s::NT, smem);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "shard_kernel occupancy");
  const long long items = (long long)a.B * a.G;
  const int grid = (int)std::min<long long>(items, (long long)std::max(occ, 1) * ctx->num_sms);
  c4s::shard_kernel<<<grid, c4s::NT, smem, (cudaStream_t)stream>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(ctx, e, "shard_kernel launch");
  return C4S_OK;
}

// cuTensorMapEncodeTiled from the driver, through the runtime (no -lcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D bf16 tensor map of `outer` rows of `inner` elements (row pitch
// row_bytes), read in 64 x 128 boxes with the 128-byte swizzle the UMMA
// descriptors expect; rows past the end read as zeros.
bool encode_bf16_rows(CUtensorMap* m, const void* base, unsigned long long inner, unsigned long long outer,
                      unsigned long long row_bytes) {
  const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)c4s::HG_BK, (cuuint32_t)c4s::HG_BM};
  cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int launch_head(c4s_ctx* ctx, const uint16_t* d_hidden, int B, int d, long long ld_hidden, const float* d_gamma,
                const float* d_beta, float eps, const uint16_t* d_weight, int N, long long ld_weight,
                const float* d_bias, uint16_t* d_norm, float* d_logits, long long ld_logits, void* stream) {
  if (!ctx) return C4S_ERR_INVALID;
  if (B < 1 || N < 1) return fail(ctx, C4S_ERR_INVALID, "B and N must be >= 1");
  if (d < c4s::HG_BK || d % c4s::HG_BK || d > c4s::HN_MAXD) return fail(ctx, C4S_ERR_INVALID, "d must be a multiple of 64 in [64, 8192]");
  if (d_norm && d % 128) return fail(ctx, C4S_ERR_INVALID, "the LayerNorm needs d a multiple of 128");
  if (ld_hidden < d || ld_weight < d || ld_logits < N) return fail(ctx, C4S_ERR_INVALID, "row stride below the row length");
  if (!d_hidden || !d_weight || !d_logits) return fail(ctx, C4S_ERR_INVALID, "null pointer");
  if (((uintptr_t)d_weight & 15) || ((ld_weight * 2) & 15) || ((uintptr_t)d_norm & 15) || ((uintptr_t)d_logits & 3))
    return fail(ctx, C4S_ERR_INVALID, "misaligned pointer or stride (TMA needs 16-byte rows)");
  if (d_norm ? (((uintptr_t)d_hidden & 7) || (ld_hidden & 3)) : (((uintptr_t)d_hidden & 15) || ((ld_hidden * 2) & 15)))
    return fail(ctx, C4S_ERR_INVALID, "misaligned hidden states");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, C4S_ERR_CUDA, "cannot select the context's device");
  const cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e;
  const uint16_t* A = d_hidden;
  long long lda = ld_hidden;
  if (d_norm) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((B + c4s::HN_WARPS - 1) / c4s::HN_WARPS));
    cfg.blockDim = dim3(32 * c4s::HN_WARPS);
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, c4s::ln_kernel, (const unsigned short*)d_hidden, ld_hidden, B, d, d_gamma, d_beta,
                           eps, (unsigned short*)d_norm);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "layer-norm kernel launch");
    A = d_norm;
    lda = d;
  }
  CUtensorMap ta, tb;
  if (!encode_bf16_rows(&ta, A, (unsigned long long)d, (unsigned long long)B, (unsigned long long)lda * 2) ||
      !encode_bf16_rows(&tb, d_weight, (unsigned long long)d, (unsigned long long)N, (unsigned long long)ld_weight * 2))
    return fail(ctx, C4S_ERR_CUDA, "tensor map encoding failed");
  c4s::HeadGemmArgs g{d_logits, ld_logits, d_bias, B, N, d, ctx->d_err};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((N + c4s::HG_BN - 1) / c4s::HG_BN), (unsigned)((B + c4s::HG_BM - 1) / c4s::HG_BM));
  cfg.blockDim = dim3(c4s::HG_THREADS);
  cfg.dynamicSmemBytes = c4s::HG_SMEM;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, c4s::head_gemm_kernel, ta, tb, g);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "head GEMM launch");
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
  return c4s_create_sized(out, max_vocab, c4s::K_CHUNK, device);
}

int c4s_create_sized(c4s_ctx** out, int32_t max_vocab, int32_t max_rows, int32_t device) {
  if (!out) return C4S_ERR_INVALID;
  *out = nullptr;
  if (max_vocab < 1 || max_vocab > c4s::MAX_VOCAB || max_rows < 1 || device < 0) return C4S_ERR_INVALID;
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
  // The attribute belongs to the kernel on the current device and is set on
  // every create for the largest row any context may launch, so contexts of
  // different sizes (and on different devices) coexist.
  const size_t smem_max = c4s::layout_for(c4s::MAX_VOCAB).total;
  e = cudaFuncSetAttribute(c4s::rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_max);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(c4s::defer_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_max);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(c4s::list_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c4s::LIST_SMEM);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(c4s::shard_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)c4s::shard_smem_bytes(c4s::MAX_VOCAB));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(c4s::fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)c4s::fused_smem_bytes(c4s::F_MAXV));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(c4s::head_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c4s::HG_SMEM);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(c4s::fused_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             (int)cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(c4s::fused_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)c4s::fused_smem_bytes(c4s::F_MAXV));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(c4s::fused_mid_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)c4s::fused_smem_bytes(c4s::F_MAXV));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(c4s::fused_mid_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             (int)cudaSharedmemCarveoutMaxShared);
  // the row kernel keeps five rows in flight per SM only with the largest
  // shared-memory carveout
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(c4s::row_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             (int)cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(c4s::list_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             (int)cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) { delete ctx; return C4S_ERR_CUDA; }
  int p2 = 1;
  while (p2 < max_vocab) p2 <<= 1;
  // one slab holds a sort of a whole row (general path, exact fallbacks) or
  // the fused kernel's long candidate list
  ctx->scratch_stride = std::max(p2, c4s::F_MIN_SCRATCH_STRIDE);
  // sized for max_rows rows per call (larger batches still run, in chunks and
  // with fewer CTAs): two slabs per fused-kernel CTA, one list per chunk row
  ctx->scratch_ctas = (int)std::min<long long>((long long)ctx->num_sms * 8, 2LL * max_rows);
  ctx->chunk = std::min(c4s::K_CHUNK, (max_rows + 31) / 32 * 32);
  e = cudaMalloc(&ctx->d_scratch, (size_t)ctx->scratch_ctas * ctx->scratch_stride * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMalloc(&ctx->d_err, sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMalloc(&ctx->d_counters, C4S_NUM_COUNTERS * sizeof(unsigned long long));
  const size_t nl = (size_t)ctx->chunk * c4s::LCAP;
  if (e == cudaSuccess) e = cudaMalloc(&ctx->d_jobs, (size_t)ctx->chunk * sizeof(c4s::RowJob));
  if (e == cudaSuccess) e = cudaMalloc(&ctx->d_lkeys, nl * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMalloc(&ctx->d_lsb, nl * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMalloc(&ctx->d_defer_rows, (1 + c4s::LIST_CLASSES) * (size_t)ctx->chunk * sizeof(int));
  if (e == cudaSuccess) e = cudaMalloc(&ctx->d_order, c4s::ROW_CLASSES * (size_t)ctx->chunk * sizeof(int));
  if (e == cudaSuccess) e = cudaMalloc(&ctx->d_defer_cnt, (c4s::FUSED_CNT + 2) * sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemset(ctx->d_defer_cnt, 0, (c4s::FUSED_CNT + 2) * sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMalloc(&ctx->d_default_params, sizeof(c4s_row_params));
  if (e == cudaSuccess) e = cudaMemset(ctx->d_default_params, 0, sizeof(c4s_row_params));
  if (e == cudaSuccess) e = cudaMemset(ctx->d_err, 0, sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemset(ctx->d_counters, 0, C4S_NUM_COUNTERS * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    free_all(ctx);
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
    free_all(ctx);
  }
  delete ctx;
  return C4S_OK;
}

const char* c4s_last_error(const c4s_ctx* ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

int c4s_set_debug(c4s_ctx* ctx, int32_t flags) {
  if (!ctx) return C4S_ERR_INVALID;
  if (flags & ~(C4S_DEBUG_FORCE_EXACT | C4S_DEBUG_FORCE_BINS | C4S_DEBUG_FORCE_REFINE | C4S_DEBUG_SPLIT_PATH |
                C4S_DEBUG_FAIL_AFTER_ROW | C4S_DEBUG_FUSED_PATH))
    return fail(ctx, C4S_ERR_INVALID, "unknown debug flag");
  ctx->debug = flags;
  return C4S_OK;
}

int c4s_kernel_timing(c4s_ctx* ctx, int32_t enable) {
  if (!ctx) return C4S_ERR_INVALID;
  ctx->timing = enable != 0;
  return C4S_OK;
}

int c4s_kernel_times(c4s_ctx* ctx, double* ms, int64_t* launches, int32_t reset) {
  if (!ctx || !ms || !launches) return C4S_ERR_INVALID;
  DeviceGuard dg(ctx->device);
  for (int k = 0; k < C4S_NUM_KERNEL_TIMERS; ++k) { ms[k] = 0.0; launches[k] = 0; }
  for (size_t c = 0; c + TEV <= ctx->tev_used; c += TEV) {
    const unsigned mask = ctx->tev_mask[c / TEV];
    for (int k = 0; k < C4S_NUM_KERNEL_TIMERS; ++k) {
      if (cudaEventSynchronize(ctx->tev[c + k + 1]) != cudaSuccess) return fail(ctx, C4S_ERR_CUDA, "timing event");
      if (!(mask & (1u << k))) continue;
      float t = 0.0f;
      if (cudaEventElapsedTime(&t, ctx->tev[c + k], ctx->tev[c + k + 1]) != cudaSuccess)
        return fail(ctx, C4S_ERR_CUDA, "timing event");
      ms[k] += t;
      launches[k] += 1;
    }
  }
  if (reset) {
    ctx->tev_used = 0;
    ctx->tev_mask.clear();
  }
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

int c4s_sample_windows(c4s_ctx* ctx, const float* d_logits, int32_t B, int32_t V, int64_t ld, const int32_t* d_hist,
                       const int64_t* d_hist_start, const int32_t* d_hist_len, int64_t hist_total,
                       const c4s_row_params* d_params, int32_t params_stride, uint64_t* d_rng,
                       const uint8_t* d_active, int32_t* d_out_ids, float* d_out_logits, int64_t out_ld,
                       void* stream) {
  int rc = check_common(ctx, B, V, ld);
  if (rc) return rc;
  if (B == 0) return C4S_OK;
  if (!d_logits || !d_params || !d_rng || !d_out_ids) return fail(ctx, C4S_ERR_INVALID, "null pointer");
  if (params_stride != 0 && params_stride != 1) return fail(ctx, C4S_ERR_INVALID, "params_stride not 0/1");
  if ((d_hist_start == nullptr) != (d_hist_len == nullptr))
    return fail(ctx, C4S_ERR_INVALID, "history windows need both starts and lengths");
  if (d_hist_start && (!d_hist && hist_total > 0)) return fail(ctx, C4S_ERR_INVALID, "history ids missing");
  if (hist_total < 0) return fail(ctx, C4S_ERR_INVALID, "hist_total < 0");
  if (d_out_logits && out_ld < V) return fail(ctx, C4S_ERR_INVALID, "out_ld < V");
  if (((uintptr_t)d_logits & 3) || (d_out_logits && ((uintptr_t)d_out_logits & 3)) || ((uintptr_t)d_hist_len & 3))
    return fail(ctx, C4S_ERR_INVALID, "misaligned pointer");
  c4s::Args a{};
  a.logits = d_logits;
  a.B = B; a.V = V; a.ld = ld;
  a.hist = d_hist; a.hist_off = reinterpret_cast<const long long*>(d_hist_start); a.hist_len = d_hist_len;
  a.hist_total = hist_total;
  a.params = d_params; a.params_stride = params_stride;
  a.rng = reinterpret_cast<unsigned long long*>(d_rng);
  a.active = d_active;
  a.out_ids = d_out_ids;
  a.out_logits = d_out_logits; a.out_ld = out_ld;
  a.mode = c4s::MODE_SAMPLE;
  return launch_rows(ctx, a, stream);
}

int c4s_decode_step(c4s_ctx* ctx, const int32_t* d_ids, int32_t B, uint8_t* d_active, int32_t stop_token,
                    int32_t* d_hist, const int64_t* d_hist_start, int32_t* d_hist_len, int32_t hist_cap,
                    const uint16_t* d_emb, int32_t n_emb, const uint16_t* d_pos_emb, int32_t D,
                    uint16_t* d_next_emb, const uint16_t* d_cur, uint16_t* d_latents, uint32_t* d_done_count,
                    void* stream) {
  if (!ctx) return C4S_ERR_INVALID;
  if (B < 0 || D < 1 || hist_cap < 0 || n_emb < 1) return fail(ctx, C4S_ERR_INVALID, "bad size");
  if (B == 0) return C4S_OK;
  if (!d_ids || !d_hist || !d_hist_start || !d_hist_len || !d_emb || !d_pos_emb || !d_next_emb || !d_done_count)
    return fail(ctx, C4S_ERR_INVALID, "null pointer");
  if ((d_latents != nullptr) != (d_cur != nullptr)) return fail(ctx, C4S_ERR_INVALID, "latents need the hidden states");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, C4S_ERR_CUDA, "cannot select the context's device");
  c4s::DecodeArgs g{d_ids, B, d_active, stop_token, d_hist, reinterpret_cast<const long long*>(d_hist_start),
                    d_hist_len, hist_cap, d_emb, n_emb, d_pos_emb, D, d_next_emb, d_cur, d_latents, d_done_count,
                    ctx->d_err};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)B);
  cfg.blockDim = dim3(c4s::DEC_NT);
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, c4s::decode_step_kernel, g);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "decode step launch");
  return C4S_OK;
}

int c4s_quantize_affine(c4s_ctx* ctx, const float* d_w, int32_t N, int32_t K, int32_t group, int32_t bits,
                        uint32_t* d_q, float* d_scales, float* d_biases, void* stream) {
  if (!ctx) return C4S_ERR_INVALID;
  if (N < 1 || K < 1 || (bits != 4 && bits != 8) || (group != 32 && group != 64 && group != 128) || K % group)
    return fail(ctx, C4S_ERR_INVALID, "need bits 4 or 8, group 32/64/128 dividing K");
  if (!d_w || !d_q || !d_scales || !d_biases) return fail(ctx, C4S_ERR_INVALID, "null pointer");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, C4S_ERR_CUDA, "cannot select the context's device");
  const long long groups = (long long)N * (K / group);
  c4s::quantize_kernel<<<(unsigned)((groups + 7) / 8), 256, 0, (cudaStream_t)stream>>>(d_w, N, K, group, bits, d_q,
                                                                                      d_scales, d_biases);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? C4S_OK : cuda_fail(ctx, e, "quantize launch");
}

int c4s_qgemv(c4s_ctx* ctx, const float* d_x, int32_t B, int32_t K, const uint32_t* d_q, const float* d_scales,
              const float* d_biases, int32_t N, int32_t group, int32_t bits, const float* d_bias_out, float* d_y,
              void* stream) {
  if (!ctx) return C4S_ERR_INVALID;
  if (B < 0 || N < 1 || K < 1 || K > c4s::QG_MAXK || (bits != 4 && bits != 8) ||
      (group != 32 && group != 64 && group != 128) || K % group || K % (128 / bits))
    return fail(ctx, C4S_ERR_INVALID, "need bits 4 or 8, group 32/64/128 dividing K, K <= 8192");
  if (B == 0) return C4S_OK;
  if (!d_x || !d_q || !d_scales || !d_biases || !d_y) return fail(ctx, C4S_ERR_INVALID, "null pointer");
  if ((uintptr_t)d_q & 15) return fail(ctx, C4S_ERR_INVALID, "packed weights must be 16-byte aligned");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, C4S_ERR_CUDA, "cannot select the context's device");
  c4s::QGemvArgs g{d_x, B, K, N, group, bits, group == 32 ? 5 : group == 64 ? 6 : 7, d_q, d_scales, d_biases,
                   d_bias_out, d_y};
  if (B == 1 && bits == 8 && ((uintptr_t)d_x & 15) == 0) {
    // the decode case: no staging of x (qgemv1_kernel)
    const int grid = (int)std::min<long long>((N + c4s::QG_WARPS - 1) / c4s::QG_WARPS, 8LL * ctx->num_sms);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(c4s::QG_NT);
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, c4s::qgemv1_kernel, g);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "qgemv launch");
    return C4S_OK;
  }
  const size_t smem = (size_t)std::min(B, c4s::QG_MAXB) * K * sizeof(float);
  if (ctx->qg_smem_set < smem) {
    const cudaError_t ea = cudaFuncSetAttribute(c4s::qgemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                (int)(c4s::QG_MAXB * c4s::QG_MAXK * sizeof(float)));
    if (ea != cudaSuccess) return cuda_fail(ctx, ea, "qgemv attribute");
    ctx->qg_smem_set = c4s::QG_MAXB * c4s::QG_MAXK * sizeof(float);
  }
  const int rows_per_cta = c4s::QG_WARPS;
  const int grid = (int)std::min<long long>((N + rows_per_cta - 1) / rows_per_cta, 8LL * ctx->num_sms);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(c4s::QG_NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, c4s::qgemv_kernel, g);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "qgemv launch");
  return C4S_OK;
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

int c4s_sample_static(const float* d_logits, int32_t B, int32_t V, int64_t ld, const int32_t* d_hist,
                      const int64_t* d_hist_off, int64_t hist_total, const c4s_row_params* d_params,
                      int32_t params_stride, uint64_t* d_rng, const uint8_t* d_active, int32_t* d_out_ids,
                      void* stream) {
  if (B < 0 || V < 1 || ld < V) return C4S_ERR_INVALID;
  if (V > C4S_STATIC_MAX_VOCAB) return C4S_ERR_CAPACITY;   // the scratch slabs hold next_pow2(V) keys
  if (B == 0) return C4S_OK;
  if (!d_logits || !d_params || !d_rng || !d_out_ids) return C4S_ERR_INVALID;
  if (params_stride != 0 && params_stride != 1) return C4S_ERR_INVALID;
  if (d_hist_off && (!d_hist && hist_total > 0)) return C4S_ERR_INVALID;
  if (hist_total < 0 || ((uintptr_t)d_logits & 3)) return C4S_ERR_INVALID;
  static_assert(C4S_STATIC_MAX_VOCAB == c4s::STATIC_MAX_VOCAB, "header and scratch agree");
  // Once per device, with that device current: the scratch's device address
  // and the general kernel's shared-memory attribute (no allocation).
  static std::mutex mu;
  static unsigned long long* scratch_of[64] = {};
  static unsigned long long* status_of[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return C4S_ERR_CUDA;
  unsigned long long* scratch = nullptr;
  unsigned long long* status = nullptr;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!scratch_of[dev]) {
      unsigned long long *p = nullptr, *q = nullptr;
      if (cudaGetSymbolAddress((void**)&p, c4s::g_static_scratch) != cudaSuccess) return C4S_ERR_CUDA;
      if (cudaGetSymbolAddress((void**)&q, c4s::g_static_status) != cudaSuccess) return C4S_ERR_CUDA;
      if (cudaFuncSetAttribute(c4s::rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)c4s::layout_for(c4s::MAX_VOCAB).total) != cudaSuccess)
        return C4S_ERR_CUDA;
      status_of[dev] = q;
      scratch_of[dev] = p;
    }
    scratch = scratch_of[dev];
    status = status_of[dev];
  }
  // the error flags and counters start at zero on every call
  if (cudaMemsetAsync(status, 0, sizeof(c4s::g_static_status), (cudaStream_t)stream) != cudaSuccess)
    return C4S_ERR_CUDA;
  c4s::Args a{};
  a.logits = d_logits;
  a.B = B; a.V = V; a.ld = ld;
  a.hist = d_hist; a.hist_off = reinterpret_cast<const long long*>(d_hist_off); a.hist_total = hist_total;
  a.params = d_params; a.params_stride = params_stride;
  a.rng = reinterpret_cast<unsigned long long*>(d_rng);
  a.active = d_active;
  a.out_ids = d_out_ids;
  a.mode = c4s::MODE_SAMPLE;
  int lg = 0;
  while ((1 << lg) < V) ++lg;
  a.qscale = std::ldexp(1.0, 62 - std::max(lg, 1));
  a.scratch = scratch;
  a.scratch_stride = 1 << lg;
  a.errflags = reinterpret_cast<unsigned*>(status);
  a.counters = status + 1;
  const int grid = std::min(B, c4s::STATIC_CTAS);
  c4s::rows_kernel<<<grid, c4s::NT, c4s::layout_for(V).total, (cudaStream_t)stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? C4S_OK : C4S_ERR_CUDA;
}

#ifdef C4S_TRACE
// Measurement builds only: copy out the fused kernel's phase trace and clear it.
int c4s_trace_read(long long* out, int* info) {
  constexpr size_t nt = (size_t)c4s::TR_CTAS * c4s::TR_ROWS * c4s::TR_PH, ni = (size_t)c4s::TR_CTAS * c4s::TR_ROWS;
  if (cudaMemcpyFromSymbol(out, c4s::g_trace, nt * sizeof(long long)) != cudaSuccess) return C4S_ERR_CUDA;
  if (cudaMemcpyFromSymbol(info, c4s::g_trace_info, ni * sizeof(int)) != cudaSuccess) return C4S_ERR_CUDA;
  static long long zl[nt];
  static int zi[ni];
  if (cudaMemcpyFromSymbol(out + nt, c4s::g_htrace, 1024 * 8 * sizeof(long long)) != cudaSuccess) return C4S_ERR_CUDA;
  if (cudaMemcpyToSymbol(c4s::g_trace, zl, sizeof(zl)) != cudaSuccess) return C4S_ERR_CUDA;
  if (cudaMemcpyToSymbol(c4s::g_trace_info, zi, sizeof(zi)) != cudaSuccess) return C4S_ERR_CUDA;
  return C4S_OK;
}
#endif

int c4s_test_div_rn(const float* d_x, float d, float* d_out, int64_t n, void* stream) {
  if (n < 0 || (n > 0 && (!d_x || !d_out))) return C4S_ERR_INVALID;
  if (n == 0) return C4S_OK;
  const long long blocks = (n + 255) / 256;
  if (blocks > 0x7fffffffLL) return C4S_ERR_INVALID;
  c4s::div_test_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(d_x, d, d_out, n);
  return cudaGetLastError() == cudaSuccess ? C4S_OK : C4S_ERR_CUDA;
}

int c4s_shard_candidates(c4s_ctx* ctx, const float* d_logits, int32_t B, int32_t V_shard, int64_t ld,
                         int32_t vocab_offset, int32_t V, const int32_t* d_hist, const int64_t* d_hist_off,
                         int64_t hist_total, const c4s_row_params* d_params, int32_t params_stride,
                         const uint8_t* d_active, c4s_candidate* d_cand, void* stream) {
  if (!ctx) return C4S_ERR_INVALID;
  if (B < 0) return fail(ctx, C4S_ERR_INVALID, "B < 0");
  if (V_shard < c4s::SHARD_CAND) return fail(ctx, C4S_ERR_INVALID, "V_shard < 64");
  if (V_shard > c4s::MAX_VOCAB) return fail(ctx, C4S_ERR_CAPACITY, "V_shard above 32768");
  if (vocab_offset < 0 || (int64_t)vocab_offset + V_shard > V)
    return fail(ctx, C4S_ERR_INVALID, "shard outside [0, V)");
  if (ld < V_shard) return fail(ctx, C4S_ERR_INVALID, "ld < V_shard");
  if (B == 0) return C4S_OK;
  if (!d_logits || !d_params || !d_cand) return fail(ctx, C4S_ERR_INVALID, "null pointer");
  if (params_stride != 0 && params_stride != 1) return fail(ctx, C4S_ERR_INVALID, "params_stride not 0/1");
  if (d_hist_off && (!d_hist && hist_total > 0)) return fail(ctx, C4S_ERR_INVALID, "history ids missing");
  if (hist_total < 0) return fail(ctx, C4S_ERR_INVALID, "hist_total < 0");
  if (((uintptr_t)d_logits & 3) || ((uintptr_t)d_cand & 7)) return fail(ctx, C4S_ERR_INVALID, "misaligned pointer");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, C4S_ERR_CUDA, "cannot select the context's device");
  c4s::ShardArgs a{};
  a.logits = d_logits;
  a.B = B; a.Vs = V_shard; a.ld = ld; a.voff = vocab_offset; a.Vtot = V;
  a.hist = d_hist; a.hist_off = reinterpret_cast<const long long*>(d_hist_off); a.hist_total = hist_total;
  a.params = d_params; a.params_stride = params_stride;
  a.active = d_active;
  a.cand = d_cand;
  a.G = 1;
  a.cand_stride = 0;
  a.errflags = ctx->d_err;
  return launch_shard(ctx, a, stream);
}

int c4s_shard_candidates_split(c4s_ctx* ctx, const float* d_logits, int32_t B, int32_t V, int64_t ld,
                               int32_t num_shards, const int32_t* d_hist, const int64_t* d_hist_off,
                               int64_t hist_total, const c4s_row_params* d_params, int32_t params_stride,
                               const uint8_t* d_active, c4s_candidate* d_cand, int64_t shard_stride,
                               void* stream) {
  return c4s_shard_candidates_sub(ctx, d_logits, B, V, ld, 0, V, num_shards, d_hist, d_hist_off, hist_total,
                                  d_params, params_stride, d_active, d_cand, shard_stride, stream);
}

int c4s_shard_candidates_sub(c4s_ctx* ctx, const float* d_logits, int32_t B, int32_t V_shard, int64_t ld,
                             int32_t vocab_offset, int32_t V, int32_t num_shards, const int32_t* d_hist,
                             const int64_t* d_hist_off, int64_t hist_total, const c4s_row_params* d_params,
                             int32_t params_stride, const uint8_t* d_active, c4s_candidate* d_cand,
                             int64_t shard_stride, void* stream) {
  if (!ctx) return C4S_ERR_INVALID;
  if (B < 0) return fail(ctx, C4S_ERR_INVALID, "B < 0");
  if (num_shards < 1 || num_shards > c4s::MAX_SHARDS) return fail(ctx, C4S_ERR_INVALID, "num_shards outside [1, 16]");
  if (V_shard < 1 || V_shard / num_shards < c4s::SHARD_CAND) return fail(ctx, C4S_ERR_INVALID, "a shard narrower than 64");
  if (vocab_offset < 0 || (int64_t)vocab_offset + V_shard > V)
    return fail(ctx, C4S_ERR_INVALID, "shard outside [0, V)");
  const int widest = V_shard / num_shards + (V_shard % num_shards ? 1 : 0);
  if (widest > c4s::MAX_VOCAB) return fail(ctx, C4S_ERR_CAPACITY, "a shard wider than 32768");
  if (ld < V_shard) return fail(ctx, C4S_ERR_INVALID, "ld < V_shard");
  if (B == 0) return C4S_OK;
  if (shard_stride < (int64_t)B * c4s::SHARD_CAND) return fail(ctx, C4S_ERR_INVALID, "shard_stride < B * 64");
  if (!d_logits || !d_params || !d_cand) return fail(ctx, C4S_ERR_INVALID, "null pointer");
  if (params_stride != 0 && params_stride != 1) return fail(ctx, C4S_ERR_INVALID, "params_stride not 0/1");
  if (d_hist_off && (!d_hist && hist_total > 0)) return fail(ctx, C4S_ERR_INVALID, "history ids missing");
  if (hist_total < 0) return fail(ctx, C4S_ERR_INVALID, "hist_total < 0");
  if (((uintptr_t)d_logits & 3) || ((uintptr_t)d_cand & 7)) return fail(ctx, C4S_ERR_INVALID, "misaligned pointer");
  c4s::ShardArgs a{};
  a.logits = d_logits;
  a.B = B; a.Vs = widest; a.ld = ld; a.voff = vocab_offset; a.Vtot = V_shard;
  a.hist = d_hist; a.hist_off = reinterpret_cast<const long long*>(d_hist_off); a.hist_total = hist_total;
  a.params = d_params; a.params_stride = params_stride;
  a.active = d_active;
  a.cand = d_cand;
  a.G = num_shards;
  a.cand_stride = shard_stride;
  a.errflags = ctx->d_err;
  return launch_shard(ctx, a, stream);
}

int c4s_merge_candidates(c4s_ctx* ctx, const c4s_candidate* d_cand, int32_t num_shards, int64_t shard_stride,
                         int32_t B, int32_t V, const c4s_row_params* d_params, int32_t params_stride,
                         uint64_t* d_rng, const uint8_t* d_active, int32_t* d_out_ids, void* stream) {
  if (!ctx) return C4S_ERR_INVALID;
  if (B < 0) return fail(ctx, C4S_ERR_INVALID, "B < 0");
  if (num_shards < 1 || num_shards > c4s::MAX_SHARDS) return fail(ctx, C4S_ERR_INVALID, "num_shards outside [1, 16]");
  if (V < 1) return fail(ctx, C4S_ERR_INVALID, "V < 1");
  if (B == 0) return C4S_OK;
  if (num_shards > 1 && shard_stride < (int64_t)B * c4s::SHARD_CAND)
    return fail(ctx, C4S_ERR_INVALID, "shard_stride < B * 64");
  if (!d_cand || !d_params || !d_rng || !d_out_ids) return fail(ctx, C4S_ERR_INVALID, "null pointer");
  if (params_stride != 0 && params_stride != 1) return fail(ctx, C4S_ERR_INVALID, "params_stride not 0/1");
  if ((uintptr_t)d_cand & 7) return fail(ctx, C4S_ERR_INVALID, "misaligned pointer");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, C4S_ERR_CUDA, "cannot select the context's device");
  c4s::MergeArgs a{};
  a.cand = d_cand;
  a.G = num_shards; a.B = B; a.Vtot = V; a.shard_stride = shard_stride;
  a.params = d_params; a.params_stride = params_stride;
  a.rng = reinterpret_cast<unsigned long long*>(d_rng);
  a.active = d_active;
  a.out_ids = d_out_ids;
  a.errflags = ctx->d_err;
  const int grid = (int)std::min<long long>((long long)B, 8LL * ctx->num_sms);
  c4s::merge_kernel<<<grid, c4s::NT, 0, (cudaStream_t)stream>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(ctx, e, "merge_kernel launch");
  return C4S_OK;
}

int c4s_head_logits(c4s_ctx* ctx, const uint16_t* d_hidden, int32_t B, int32_t d, int64_t ld_hidden,
                    const float* d_gamma, const float* d_beta, float eps, const uint16_t* d_weight, int32_t N,
                    int64_t ld_weight, const float* d_bias, uint16_t* d_norm, float* d_logits, int64_t ld_logits,
                    void* stream) {
  return launch_head(ctx, d_hidden, B, d, ld_hidden, d_gamma, d_beta, eps, d_weight, N, ld_weight, d_bias, d_norm,
                     d_logits, ld_logits, stream);
}

int c4s_head_sample(c4s_ctx* ctx, const uint16_t* d_hidden, int32_t B, int32_t d, int64_t ld_hidden,
                    const float* d_gamma, const float* d_beta, float eps, const uint16_t* d_weight, int32_t N,
                    int64_t ld_weight, const float* d_bias, uint16_t* d_norm, float* d_logits, int64_t ld_logits,
                    const int32_t* d_hist, const int64_t* d_hist_off, int64_t hist_total,
                    const c4s_row_params* d_params, int32_t params_stride, uint64_t* d_rng, const uint8_t* d_active,
                    int32_t* d_out_ids, void* stream) {
  if (!ctx) return C4S_ERR_INVALID;
  if (N > ctx->max_vocab) return fail(ctx, C4S_ERR_CAPACITY, "N above the context's max_vocab");
  const int rc = launch_head(ctx, d_hidden, B, d, ld_hidden, d_gamma, d_beta, eps, d_weight, N, ld_weight, d_bias,
                             d_norm, d_logits, ld_logits, stream);
  if (rc) return rc;
  return c4s_sample(ctx, d_logits, B, N, ld_logits, d_hist, d_hist_off, hist_total, d_params, params_stride, d_rng,
                    d_active, d_out_ids, nullptr, 0, stream);
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
  if (err & C4S_DEVERR_HIST_RANGE) return fail(ctx, C4S_ERR_DEVICE, "history offsets out of range");
  if (err & C4S_DEVERR_HIST_FULL)
    return fail(ctx, C4S_ERR_DEVICE, "a decode step found a full history window (the row stopped)");
  if (err & C4S_DEVERR_SHARD)
    return fail(ctx, C4S_ERR_DEVICE, "vocab-sharded merge refused rows it cannot decide exactly (id -1)");
  if (err) return fail(ctx, C4S_ERR_DEVICE, "unknown device error flag");
  return C4S_OK;
}

}  // extern "C"
