/*
 * c4s_oracle.h -- CPU oracle for the T2S sampling stage.
 *
 * TEST INFRASTRUCTURE ONLY. This is a plain-C restatement of the reference's
 * sampling processors and inline categorical draw, used by tests/, by
 * __graft_entry__.smoke() and by bench.py's CPU-baseline leg as the checker.
 * The product path (the CUDA library) never links or calls it.
 *
 * Pinned against: the reference's HuggingFace golden vectors (tests/golden,
 * made by tools/dump_golden.py:807-825 of the reference) and the unmodified
 * reference src/t2s/sampling.cpp compiled from source into oracle/_ref/.
 */
#ifndef C4S_ORACLE_H_
#define C4S_ORACLE_H_

#include <stdint.h>

#include "../include/c4s_sampling.h"

#ifdef __cplusplus
extern "C" {
#endif

/* sampling.cpp:14-17 */
void c4o_temperature(float* x, int32_t n, float temp);
/* sampling.cpp:19-28 */
void c4o_repetition_penalty(float* x, int32_t n, const int32_t* hist,
                            int64_t h, float penalty);
/* sampling.cpp:30-40 */
void c4o_top_k(float* x, int32_t n, int32_t k);
/* sampling.cpp:42-71, ties ordered by ascending index */
void c4o_top_p(float* x, int32_t n, float p, int32_t min_keep);
/* sampling.cpp:73-76 */
int32_t c4o_argmax(const float* x, int32_t n);
/* text2semantic.cpp:150-165 (and :315-331): advances *state once */
int32_t c4o_draw(const float* x, int32_t n, uint64_t* state);

/* Diagnostics for parity tests (no reference counterpart).
 * c4o_top_p_info: for the top-p decision on x (already tempered / top-k'd),
 * reports whether the removal boundary splits a group of equal values (where
 * the reference's unstable std::sort leaves the outcome unspecified) and the
 * smallest |cum_j - (1-p)| over the two positions around the boundary.     */
void c4o_top_p_info(const float* x, int32_t n, float p, int32_t min_keep,
                    int32_t* tie_at_boundary, double* margin);

/* text2semantic.cpp:109 / :292-295 */
void c4o_seed_states(uint64_t* s, int32_t B, uint64_t seed, int64_t row_offset);

/* One row of text2semantic.cpp:303-331 on a private copy; writes the
 * processed logits to out_row (may be NULL). Returns the token id. */
int32_t c4o_sample_row(const float* row, int32_t V, const int32_t* hist,
                       int64_t h, const c4s_row_params* P, uint64_t* state,
                       float* out_row);

/* Batched mirror of c4s_sample() (same argument meaning, host pointers). */
void c4o_sample_batch(const float* logits, int32_t B, int32_t V, int64_t ld,
                      const int32_t* hist, const int64_t* hist_off,
                      const c4s_row_params* params, int32_t params_stride,
                      uint64_t* rng, const uint8_t* active, int32_t* out_ids,
                      float* out_logits, int64_t out_ld, int32_t nthreads);

/* Batched mirror of c4s_process() (in place). */
void c4o_process_batch(float* logits, int32_t B, int32_t V, int64_t ld,
                       const int32_t* hist, const int64_t* hist_off,
                       const c4s_row_params* params, int32_t params_stride,
                       int32_t stages, int32_t nthreads);

/* Batched argmax. */
void c4o_argmax_batch(const float* logits, int32_t B, int32_t V, int64_t ld,
                      int32_t* out_ids);

#ifdef __cplusplus
}
#endif

#endif /* C4S_ORACLE_H_ */
