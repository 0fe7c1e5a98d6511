// c4s_qgemv.cuh -- quantized decode GEMVs of the T2S GPT-2 (sm_100a).
//
// The reference's product default (apps/c4tts_cli.cpp:300-306: C4TTS_QUANT=8)
// quantizes every GPT-2 projection weight once (gpt2.cpp:52-60: the (out, in)
// transpose of the Conv1D weight, mx::quantize with group 64) and runs each
// decode projection as mx::quantized_matmul(x, w_q, scales, biases,
// transpose=true) + bias (gpt2.cpp:61-63). MLX (pinned at v0.31.2 by the
// reference's CMakeLists.txt:46) is not present; its published affine scheme
// is: per group of `group` consecutive elements of a weight row,
//     scale = (max - min) / (2^bits - 1),  bias = min,
//     q = round((w - bias) / scale)  in [0, 2^bits - 1],
//     w ~= scale * q + bias,
// q packed little-end-first into 32-bit words (4 per word at 8 bits, 8 at 4).
//
// quantize_kernel builds that layout on the device (one warp per group).
// qgemv_kernel computes y[b, n] = sum_k x[b, k] (scale q + bias)[n, k] + bo[n]
// for a decode batch of up to QG_MAXB rows: each warp streams one weight row
// at a time with 16-byte loads (512 contiguous bytes per warp instruction),
// every lane dequantizes its 16 (8-bit) or 32 (4-bit) weights exactly in fp32
// (q as a float is exact; scale q + bias by one FMA) and accumulates against
// x, which the CTA stages in shared memory once. The weight stream is the
// roofline: (bits/8 + 8/group) bytes per weight.
#pragma once

namespace c4s {

constexpr int QG_NT = 256;
constexpr int QG_WARPS = QG_NT / 32;
constexpr int QG_MAXB = 4;                         // decode rows per pass over the weights
constexpr int QG_MAXK = 8192;                      // x rows staged in shared memory (QG_MAXB x QG_MAXK fp32)

struct QGemvArgs {
  const float* x;        // [B, K]
  int B, K, N, group, bits;
  int glog;              // log2(group)
  const unsigned* q;     // [N, K * bits / 32]
  const float* scales;   // [N, K / group]
  const float* biases;   // [N, K / group]
  const float* bias_out; // [N] or null
  float* y;              // [B, N]
};

// x in shared memory is laid out by position inside a chunk: element k of
// row b (chunk c = k / per, position i = k % per) sits at b K + i nchunk + c,
// so the lanes of a warp, which work consecutive chunks, read consecutive
// words.
// 16 bytes of 8-bit codes (one lane's chunk c) times x, for each decode row.
template <int NB>
__device__ __forceinline__ void qdot8(const uint4 w, float s, float bi, const float* xs, int K, int nchunk, int c,
                                      float (&acc)[QG_MAXB]) {
  const unsigned word[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float qf = (float)((word[j] >> (8 * e)) & 0xffu);
      const float wv = fmaf(s, qf, bi);
#pragma unroll
      for (int b = 0; b < NB; ++b) acc[b] = fmaf(xs[b * K + (4 * j + e) * nchunk + c], wv, acc[b]);
    }
  }
}

// 16 bytes of 4-bit codes (32 weights): the group's scale and bias may
// change inside the chunk when group < 32 (looked up per 8-weight word).
template <int NB>
__device__ __forceinline__ void qdot4(const uint4 w, const float* srow, const float* brow, int glog,
                                      const float* xs, int K, int nchunk, int c, float (&acc)[QG_MAXB]) {
  const unsigned word[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int kg = (32 * c + 8 * j) >> glog;
    const float s = __ldg(srow + kg), bi = __ldg(brow + kg);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float qf = (float)((word[j] >> (4 * e)) & 0xfu);
      const float wv = fmaf(s, qf, bi);
#pragma unroll
      for (int b = 0; b < NB; ++b) acc[b] = fmaf(xs[b * K + (8 * j + e) * nchunk + c], wv, acc[b]);
    }
  }
}

constexpr int QG_INFLIGHT = 4;                     // 16-byte weight chunks a lane has in flight

template <int NB>
__device__ __forceinline__ void qgemv_rows(const QGemvArgs& g, const float* xs, int b0) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int per = 128 / g.bits;                    // weights per 16-byte chunk: 16 or 32
  const int nchunk = g.K / per;
  const int ng = g.K / g.group;
  for (int n = blockIdx.x * QG_WARPS + warp; n < g.N; n += gridDim.x * QG_WARPS) {
    const uint4* wr = reinterpret_cast<const uint4*>(g.q + (size_t)n * (g.K * g.bits / 32));
    const float* srow = g.scales + (size_t)n * ng;
    const float* brow = g.biases + (size_t)n * ng;
    float acc[QG_MAXB];
#pragma unroll
    for (int b = 0; b < QG_MAXB; ++b) acc[b] = 0.0f;
    // QG_INFLIGHT chunks per lane in flight: their loads are issued before any is used
    for (int c0 = lane; c0 < nchunk; c0 += QG_INFLIGHT * 32) {
      uint4 w[QG_INFLIGHT];
#pragma unroll
      for (int u = 0; u < QG_INFLIGHT; ++u)
        w[u] = c0 + 32 * u < nchunk ? __ldcs(wr + c0 + 32 * u) : make_uint4(0u, 0u, 0u, 0u);   // streamed once
#pragma unroll
      for (int u = 0; u < QG_INFLIGHT; ++u) {
        const int c = c0 + 32 * u;
        if (c >= nchunk) break;
        if (g.bits == 8) {
          const int kg = (c * 16) >> g.glog;       // group >= 16: a chunk lies in one group
          qdot8<NB>(w[u], __ldg(srow + kg), __ldg(brow + kg), xs, g.K, nchunk, c, acc);
        } else {
          qdot4<NB>(w[u], srow, brow, g.glog, xs, g.K, nchunk, c, acc);
        }
      }
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      float v = acc[b];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
      if (lane == 0) g.y[(size_t)(b0 + b) * g.N + n] = v + (g.bias_out ? g.bias_out[n] : 0.0f);
    }
  }
}

__global__ void __launch_bounds__(QG_NT) qgemv_kernel(QGemvArgs g) {
  extern __shared__ __align__(16) float xs[];
  grid_dep_wait();                                 // x (and the weights) come from earlier kernels
  grid_dep_launch();
  for (int b0 = 0; b0 < g.B; b0 += QG_MAXB) {
    const int nb = min(QG_MAXB, g.B - b0);
    __syncthreads();                               // the previous pass is done with xs
    const int plog = g.bits == 8 ? 4 : 5, nchunk = g.K >> plog;   // 16 or 32 weights per chunk
    for (int b = 0; b < nb; ++b)
      for (int k = threadIdx.x; k < g.K; k += QG_NT)
        xs[b * g.K + (k & ((1 << plog) - 1)) * nchunk + (k >> plog)] = g.x[(size_t)(b0 + b) * g.K + k];
    __syncthreads();
    switch (nb) {
      case 1: qgemv_rows<1>(g, xs, b0); break;
      case 2: qgemv_rows<2>(g, xs, b0); break;
      case 3: qgemv_rows<3>(g, xs, b0); break;
      default: qgemv_rows<4>(g, xs, b0); break;
    }
  }
}

// The decode case -- one row of x, 8-bit codes -- without the staging of x:
// each lane's chunks (16 codes = 16 B) are loaded together with the 16
// values of x they multiply (four float4 through L1; x is a few KB that every
// warp reads) and their group's scale and bias, QG_INFLIGHT chunks at a time,
// so a warp's row costs about one memory round trip instead of the staging
// pass, a CTA barrier and then the weights. The products are summed in the
// same order as qgemv_rows (per lane: chunks in order, the 16 weights of a
// chunk in order; then the warp's shuffle tree). Needs x 16-byte aligned.
__global__ void __launch_bounds__(QG_NT, 2) qgemv1_kernel(QGemvArgs g) {
  grid_dep_wait();                                 // x comes from the previous kernel
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nchunk = g.K >> 4;                     // 16 codes per chunk
  const int ng = g.K >> g.glog;
  const float4* x4 = reinterpret_cast<const float4*>(g.x);
  for (int n = blockIdx.x * QG_WARPS + warp; n < g.N; n += gridDim.x * QG_WARPS) {
    const uint4* wr = reinterpret_cast<const uint4*>(g.q + (size_t)n * (g.K / 4));
    const float* srow = g.scales + (size_t)n * ng;
    const float* brow = g.biases + (size_t)n * ng;
    float acc = 0.0f;
    for (int c0 = lane; c0 < nchunk; c0 += QG_INFLIGHT * 32) {
      uint4 w[QG_INFLIGHT];
      float4 xv[QG_INFLIGHT][4];
      float sc[QG_INFLIGHT], bi[QG_INFLIGHT];
#pragma unroll
      for (int u = 0; u < QG_INFLIGHT; ++u) {
        const int c = c0 + 32 * u;
        const bool ok = c < nchunk;
        const int kg = (c * 16) >> g.glog;         // group >= 16: a chunk lies in one group
        w[u] = ok ? __ldcs(wr + c) : make_uint4(0u, 0u, 0u, 0u);   // streamed once
        sc[u] = ok ? __ldg(srow + kg) : 0.0f;
        bi[u] = ok ? __ldg(brow + kg) : 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) xv[u][j] = ok ? __ldg(x4 + 4 * c + j) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < QG_INFLIGHT; ++u) {
        if (c0 + 32 * u >= nchunk) break;
        const unsigned word[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float xe[4] = {xv[u][j].x, xv[u][j].y, xv[u][j].z, xv[u][j].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float wv = fmaf(sc[u], (float)((word[j] >> (8 * e)) & 0xffu), bi[u]);
            acc = fmaf(xe[e], wv, acc);
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(FULL, acc, o);
    if (lane == 0) g.y[n] = acc + (g.bias_out ? g.bias_out[n] : 0.0f);
  }
}

// Affine quantization of w [N, K] (one warp per group of <= 128 weights,
// lane l holding elements l, l + 32, ...): min / max by warp reductions,
// q = round-half-even((w - min) / scale), clamped to [0, 2^bits - 1]; a
// group with max == min gets scale 0 and q = 0 (w = bias exactly).
__global__ void __launch_bounds__(256) quantize_kernel(const float* __restrict__ w, int N, int K, int group,
                                                       int bits, unsigned* __restrict__ q,
                                                       float* __restrict__ scales, float* __restrict__ biases) {
  const int lane = threadIdx.x & 31;
  const long long gid = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int ng = K / group;
  if (gid >= (long long)N * ng) return;
  const int n = (int)(gid / ng), gi = (int)(gid % ng);
  const float* wg = w + (size_t)n * K + (size_t)gi * group;
  float v[4], mn = INFINITY, mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int e = lane + 32 * j;
    v[j] = e < group ? wg[e] : 0.0f;
    if (e < group) { mn = fminf(mn, v[j]); mx = fmaxf(mx, v[j]); }
  }
  mn = warp_reduce(mn, [](float a, float b) { return fminf(a, b); });
  mx = warp_reduce(mx, [](float a, float b) { return fmaxf(a, b); });
  const float qmax = (float)((1 << bits) - 1);
  const float scale = (mx - mn) / qmax;
  if (lane == 0) {
    scales[(size_t)n * ng + gi] = scale;
    biases[(size_t)n * ng + gi] = mn;
  }
  const int per_word = 32 / bits;
  unsigned* qr = q + ((size_t)n * K + (size_t)gi * group) / per_word;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int e = lane + 32 * j;
    unsigned code = 0u;
    if (e < group && scale > 0.0f) code = (unsigned)fminf(fmaxf(rintf((v[j] - mn) / scale), 0.0f), qmax);
    // assemble words: the per_word lanes of a word combine their codes
    unsigned part = e < group ? code << (bits * (e % per_word)) : 0u;
#pragma unroll
    for (int o = 1; o < 8; o <<= 1)
      if (o < per_word) part |= __shfl_xor_sync(FULL, part, o);
    if (e < group && e % per_word == 0) qr[e / per_word] = part;
  }
}

}  // namespace c4s
