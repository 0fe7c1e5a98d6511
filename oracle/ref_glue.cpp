// ref_glue.cpp -- C entry points around the reference's own sampling
// processors, compiled from the reference source tree (src/t2s/sampling.cpp,
// unmodified) into oracle/_ref/libc4s_ref.so.
//
// TEST INFRASTRUCTURE ONLY: used by tests/ (to pin the C oracle), by
// tests/golden/make_golden.py (to write golden fixtures) and by bench.py's
// CPU-baseline leg. The product library never links it.
//
// The processors are the reference's. The categorical draw lives inline in
// text2semantic.cpp:150-165 / :315-331, which needs MLX and cannot compile
// here, so it comes from the oracle's restatement (c4o_draw).
#include <cstdint>
#include <cstring>
#include <vector>

#include "c4tts/t2s.h"
#include "c4s_oracle.h"

namespace sp = c4::t2s::sampling;

namespace {
std::vector<float> to_vec(const float* x, int32_t n) { return std::vector<float>(x, x + n); }
void from_vec(const std::vector<float>& v, float* x) { std::memcpy(x, v.data(), v.size() * sizeof(float)); }
}  // namespace

extern "C" {

void ref_temperature(float* x, int32_t n, float t) {
  auto v = to_vec(x, n); sp::temperature(v, t); from_vec(v, x);
}
void ref_repetition_penalty(float* x, int32_t n, const int32_t* hist, int64_t h, float pen) {
  auto v = to_vec(x, n);
  std::vector<int> prev(hist, hist + h);
  sp::repetition_penalty(v, prev, pen);
  from_vec(v, x);
}
void ref_top_k(float* x, int32_t n, int32_t k) {
  auto v = to_vec(x, n); sp::top_k(v, k); from_vec(v, x);
}
void ref_top_p(float* x, int32_t n, float p, int32_t min_keep) {
  auto v = to_vec(x, n); sp::top_p(v, p, min_keep); from_vec(v, x);
}
int32_t ref_argmax(const float* x, int32_t n) {
  auto v = to_vec(x, n); return sp::argmax(v);
}

// The per-row body of text2semantic.cpp:303-331 with the reference's own
// processors; rows run on `nthreads` OpenMP threads (1 = the reference's
// serial loop).
void ref_sample_batch(const float* logits, int32_t B, int32_t V, int64_t ld,
                      const int32_t* hist, const int64_t* hist_off,
                      const c4s_row_params* params, int32_t params_stride,
                      uint64_t* rng, const uint8_t* active, int32_t* out_ids,
                      float* out_logits, int64_t out_ld, int32_t nthreads) {
#pragma omp parallel for schedule(dynamic, 4) num_threads(nthreads > 0 ? nthreads : 1)
  for (int32_t b = 0; b < B; ++b) {
    if (active && !active[b]) { out_ids[b] = -1; continue; }
    const c4s_row_params& P = params[(int64_t)b * params_stride];
    std::vector<float> v(logits + (int64_t)b * ld, logits + (int64_t)b * ld + V);
    std::vector<int> gen;
    if (hist_off) gen.assign(hist + hist_off[b], hist + hist_off[b + 1]);
    sp::repetition_penalty(v, gen, P.repetition_penalty);
    int32_t tok;
    if (P.greedy) {
      tok = sp::argmax(v);
    } else {
      sp::temperature(v, P.temperature);
      sp::top_k(v, P.top_k);
      sp::top_p(v, P.top_p, P.min_tokens_to_keep);
      tok = c4o_draw(v.data(), V, rng + b);
    }
    if (out_logits) std::memcpy(out_logits + (int64_t)b * out_ld, v.data(), sizeof(float) * V);
    out_ids[b] = tok;
  }
}

}  // extern "C"
