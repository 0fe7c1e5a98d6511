/*
 * c4s_oracle.c -- CPU oracle (plain C) for the T2S sampling stage.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for tests/, smoke() and the CPU
 * baseline of bench.py. Nothing in the product library calls this code.
 *
 * Each function restates one piece of the reference, operation for operation
 * (same float/double types, same sequential summation order, same compare
 * operators), citing the file:line it follows. Compiled with
 * -ffp-contract=off so that no multiply-add is fused.
 *
 * One deliberate choice: top_p orders equal logits by ascending index. The
 * reference uses std::sort, whose order among equal keys is unspecified; the
 * only observable effect is which of several equal logits is removed when the
 * top-p boundary falls inside such a group. c4o_top_p_info() reports when that
 * happens so tests can tell it apart from a real mismatch.
 */
#include "c4s_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define C4O_GOLDEN_STATE 0x9E3779B97F4A7C15ull /* text2semantic.cpp:109 */
#define C4O_ROW_STRIDE 0x100000001b3ull        /* text2semantic.cpp:294 */

/* sampling.cpp:14-17 */
void c4o_temperature(float* x, int32_t n, float temp) {
  if (temp == 1.0f || temp <= 0.0f) return;
  for (int32_t i = 0; i < n; ++i) x[i] /= temp;
}

/* sampling.cpp:19-28: each distinct id in [0, n) is penalised once. */
void c4o_repetition_penalty(float* x, int32_t n, const int32_t* hist,
                            int64_t h, float penalty) {
  if (penalty == 1.0f || n <= 0) return;
  unsigned char* seen = (unsigned char*)calloc((size_t)n, 1);
  for (int64_t j = 0; j < h; ++j) {
    int32_t t = hist[j];
    if (t < 0 || t >= n) continue;
    if (seen[t]) continue;
    seen[t] = 1;
    float s = x[t];
    x[t] = (s < 0) ? s * penalty : s / penalty;
  }
  free(seen);
}

static int cmp_desc_f32(const void* a, const void* b) {
  float fa = *(const float*)a, fb = *(const float*)b;
  return (fa > fb) ? -1 : (fa < fb) ? 1 : 0;
}

/* sampling.cpp:30-40: threshold = k-th largest value; v < thresh -> -inf. */
void c4o_top_k(float* x, int32_t n, int32_t k) {
  if (k <= 0 || k >= n) return;
  float* sorted = (float*)malloc(sizeof(float) * (size_t)n);
  memcpy(sorted, x, sizeof(float) * (size_t)n);
  qsort(sorted, (size_t)n, sizeof(float), cmp_desc_f32);
  const float thresh = sorted[k - 1];
  free(sorted);
  for (int32_t i = 0; i < n; ++i)
    if (x[i] < thresh) x[i] = -INFINITY;
}

/* Ascending (value, index) order for top_p. qsort needs the row: pass it
 * through a struct array instead of a global so the oracle is reentrant. */
typedef struct { float v; int32_t i; } c4o_vi;
static int cmp_asc_vi(const void* a, const void* b) {
  const c4o_vi* A = (const c4o_vi*)a;
  const c4o_vi* B = (const c4o_vi*)b;
  if (A->v < B->v) return -1;
  if (A->v > B->v) return 1;
  return (A->i < B->i) ? -1 : (A->i > B->i) ? 1 : 0;
}

/* Shared body of top_p and its diagnostics: fills remove[] (by sorted
 * position), returns the number of removed positions (a prefix). */
static int32_t top_p_core(const float* x, int32_t n, float p, int32_t min_keep,
                          c4o_vi* s, char* remove, double* cum_out) {
  for (int32_t i = 0; i < n; ++i) { s[i].v = x[i]; s[i].i = i; }
  qsort(s, (size_t)n, sizeof(c4o_vi), cmp_asc_vi);          /* :45-48 */
  float maxv = x[0];                                          /* :51    */
  for (int32_t i = 1; i < n; ++i) if (maxv < x[i]) maxv = x[i];
  double* probs = (double*)malloc(sizeof(double) * (size_t)n);
  double sum = 0;
  for (int32_t i = 0; i < n; ++i) {                           /* :54-57 */
    probs[i] = exp((double)(s[i].v - maxv));
    sum += probs[i];
  }
  double cum = 0;
  for (int32_t i = 0; i < n; ++i) {                           /* :62-65 */
    cum += probs[i] / sum;
    if (cum_out) cum_out[i] = cum;
    remove[i] = (cum <= (1.0 - p)) ? 1 : 0;
  }
  for (int32_t i = n - min_keep; i < n; ++i)                  /* :67-68 */
    if (i >= 0) remove[i] = 0;
  free(probs);
  int32_t nrem = 0;
  while (nrem < n && remove[nrem]) ++nrem;
  return nrem;
}

/* sampling.cpp:42-71 */
void c4o_top_p(float* x, int32_t n, float p, int32_t min_keep) {
  if (n <= 0) return;
  c4o_vi* s = (c4o_vi*)malloc(sizeof(c4o_vi) * (size_t)n);
  char* remove = (char*)malloc((size_t)n);
  top_p_core(x, n, p, min_keep, s, remove, NULL);
  for (int32_t i = 0; i < n; ++i)                             /* :69-70 */
    if (remove[i]) x[s[i].i] = -INFINITY;
  free(remove);
  free(s);
}

void c4o_top_p_info(const float* x, int32_t n, float p, int32_t min_keep,
                    int32_t* tie_at_boundary, double* margin) {
  *tie_at_boundary = 0;
  *margin = INFINITY;
  if (n <= 0) return;
  c4o_vi* s = (c4o_vi*)malloc(sizeof(c4o_vi) * (size_t)n);
  char* remove = (char*)malloc((size_t)n);
  double* cum = (double*)malloc(sizeof(double) * (size_t)n);
  int32_t nrem = top_p_core(x, n, p, min_keep, s, remove, cum);
  if (nrem > 0 && nrem < n && s[nrem - 1].v == s[nrem].v) *tie_at_boundary = 1;
  /* the mask prefix is a prefix of the ascending order (remove is monotone
   * except for the min_keep override); check both sides of the crossing. */
  const double thr = 1.0 - p;
  int32_t j = 0;
  while (j < n && cum[j] <= thr) ++j;
  if (j > 0) *margin = fabs(cum[j - 1] - thr);
  if (j < n) {
    double m2 = fabs(cum[j] - thr);
    if (m2 < *margin) *margin = m2;
  }
  free(cum);
  free(remove);
  free(s);
}

/* sampling.cpp:73-76 (std::max_element: first maximum) */
int32_t c4o_argmax(const float* x, int32_t n) {
  int32_t best = 0;
  for (int32_t i = 1; i < n; ++i)
    if (x[best] < x[i]) best = i;
  return best;
}

/* text2semantic.cpp:150-165 */
int32_t c4o_draw(const float* x, int32_t n, uint64_t* state) {
  float maxv = -1e30f;
  for (int32_t i = 0; i < n; ++i) maxv = (maxv < x[i]) ? x[i] : maxv;
  double* probs = (double*)malloc(sizeof(double) * (size_t)(n > 0 ? n : 1));
  double sum = 0;
  for (int32_t i = 0; i < n; ++i) {
    probs[i] = isinf(x[i]) ? 0.0 : exp((double)(x[i] - maxv));
    sum += probs[i];
  }
  uint64_t r = *state;
  r ^= r << 13; r ^= r >> 7; r ^= r << 17;
  *state = r;
  double rr = (double)(r >> 11) / (double)(1ull << 53) * sum;
  double acc = 0;
  int32_t tok = n - 1;
  for (int32_t i = 0; i < n; ++i) {
    acc += probs[i];
    if (rr <= acc) { tok = i; break; }
  }
  free(probs);
  return tok;
}

/* text2semantic.cpp:109 (row 0) and :292-295 */
void c4o_seed_states(uint64_t* s, int32_t B, uint64_t seed, int64_t row_offset) {
  const uint64_t base = seed ? seed : C4O_GOLDEN_STATE;
  for (int32_t b = 0; b < B; ++b)
    s[b] = base + (uint64_t)(row_offset + b) * C4O_ROW_STRIDE;
}

/* text2semantic.cpp:307-331: penalty, then argmax or the sample chain. */
int32_t c4o_sample_row(const float* row, int32_t V, const int32_t* hist,
                       int64_t h, const c4s_row_params* P, uint64_t* state,
                       float* out_row) {
  float* x = (float*)malloc(sizeof(float) * (size_t)(V > 0 ? V : 1));
  memcpy(x, row, sizeof(float) * (size_t)V);
  c4o_repetition_penalty(x, V, hist, h, P->repetition_penalty);
  int32_t tok;
  if (P->greedy) {
    tok = c4o_argmax(x, V);
  } else {
    c4o_temperature(x, V, P->temperature);
    c4o_top_k(x, V, P->top_k);
    c4o_top_p(x, V, P->top_p, P->min_tokens_to_keep);
    tok = c4o_draw(x, V, state);
  }
  if (out_row) memcpy(out_row, x, sizeof(float) * (size_t)V);
  free(x);
  return tok;
}

void c4o_sample_batch(const float* logits, int32_t B, int32_t V, int64_t ld,
                      const int32_t* hist, const int64_t* hist_off,
                      const c4s_row_params* params, int32_t params_stride,
                      uint64_t* rng, const uint8_t* active, int32_t* out_ids,
                      float* out_logits, int64_t out_ld, int32_t nthreads) {
  (void)nthreads;
#pragma omp parallel for schedule(dynamic, 4) num_threads(nthreads > 0 ? nthreads : 1)
  for (int32_t b = 0; b < B; ++b) {
    if (active && !active[b]) { out_ids[b] = -1; continue; }
    const int32_t* hb = hist_off ? hist + hist_off[b] : hist;
    const int64_t hn = hist_off ? hist_off[b + 1] - hist_off[b] : 0;
    out_ids[b] = c4o_sample_row(logits + (int64_t)b * ld, V, hb, hn,
                                params + (int64_t)b * params_stride, rng + b,
                                out_logits ? out_logits + (int64_t)b * out_ld : NULL);
  }
}

void c4o_process_batch(float* logits, int32_t B, int32_t V, int64_t ld,
                       const int32_t* hist, const int64_t* hist_off,
                       const c4s_row_params* params, int32_t params_stride,
                       int32_t stages, int32_t nthreads) {
  (void)nthreads;
#pragma omp parallel for schedule(dynamic, 4) num_threads(nthreads > 0 ? nthreads : 1)
  for (int32_t b = 0; b < B; ++b) {
    float* x = logits + (int64_t)b * ld;
    const c4s_row_params* P = params + (int64_t)b * params_stride;
    if ((stages & C4S_STAGE_PENALTY) && hist_off)
      c4o_repetition_penalty(x, V, hist + hist_off[b], hist_off[b + 1] - hist_off[b],
                             P->repetition_penalty);
    if (stages & C4S_STAGE_TEMPERATURE) c4o_temperature(x, V, P->temperature);
    if (stages & C4S_STAGE_TOP_K) c4o_top_k(x, V, P->top_k);
    if (stages & C4S_STAGE_TOP_P) c4o_top_p(x, V, P->top_p, P->min_tokens_to_keep);
  }
}

void c4o_argmax_batch(const float* logits, int32_t B, int32_t V, int64_t ld,
                      int32_t* out_ids) {
  for (int32_t b = 0; b < B; ++b) out_ids[b] = c4o_argmax(logits + (int64_t)b * ld, V);
}
