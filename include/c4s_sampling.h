/*
 * c4s_sampling.h -- C ABI of the B200 (sm_100a) T2S sampling stage.
 *
 * This library replaces the host-side sampling stage of the Confucius4-TTS
 * C++/MLX engine (raoqu/mlx-confucius4-tts). In the reference, every AR decode
 * step copies one 8194-wide fp32 logits row per stream to the host and runs
 *
 *     repetition_penalty -> (greedy: argmax)
 *                        -> (sample: temperature -> top_k -> top_p -> draw)
 *
 * in scalar C++ on a std::vector<float>:
 *   include/c4tts/t2s.h:82-89          declarations of the five processors
 *   src/t2s/sampling.cpp:14-76         their definitions
 *   src/t2s/text2semantic.cpp:142-165  single-stream call order + inline draw
 *   src/t2s/text2semantic.cpp:303-331  batched call order + inline draw
 *   src/t2s/text2semantic.cpp:109,294  xorshift64 state seeding
 *
 * Here the logits stay in device memory and one call processes a whole batch
 * of rows. All entry points
 *   - return 0 (C4S_OK) or a negative c4s_status, and never throw;
 *   - take caller-owned DEVICE pointers (except where noted) and a
 *     cudaStream_t passed as void*; work is stream-ordered and asynchronous;
 *   - never allocate device memory after c4s_create();
 *   - are thread-compatible: one context per host thread (or stream) at a time.
 *
 * Parity contract with the reference (same inputs, same xorshift64 state):
 *   penalised / tempered / top-k-masked logits are bit-identical; top-p masks
 *   are identical (ties at the top-p boundary are broken by ascending index,
 *   where the reference's std::sort leaves the order unspecified); sampled ids
 *   are identical. Inputs containing NaN or +inf are outside the contract
 *   (the reference's std::sort is undefined for NaN; +inf makes its softmax NaN).
 */
#ifndef C4S_SAMPLING_H_
#define C4S_SAMPLING_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define C4S_ABI_VERSION 1

/* Status codes. */
typedef enum c4s_status {
  C4S_OK = 0,
  C4S_ERR_INVALID = -1,   /* bad argument (null pointer, size, stride, mode) */
  C4S_ERR_CUDA = -2,      /* a CUDA runtime call failed; see c4s_last_error() */
  C4S_ERR_CAPACITY = -3,  /* V above the context's max_vocab / kernel limit */
  C4S_ERR_DEVICE = -4,    /* a kernel raised a device-side error flag */
  C4S_ERR_TIMEOUT = -5,   /* a bounded device wait gave up */
  C4S_ERR_NCCL = -6       /* a collective failed (vocab-sharded path) */
} c4s_status;

/* Per-row sampling parameters. One struct per row (params_stride = 1) or one
 * struct broadcast to all rows (params_stride = 0). Defaults of the reference
 * (include/c4tts/pipeline.h:26-37): T 0.8, top_k 30, top_p 0.8, penalty 10,
 * greedy 0, min_tokens_to_keep 1.                                           */
typedef struct c4s_row_params {
  float temperature;          /* sampling.cpp:14-17; skipped if ==1 or <=0     */
  int32_t top_k;              /* sampling.cpp:30-40; skipped if <=0 or >=V     */
  float top_p;                /* sampling.cpp:42-71                            */
  float repetition_penalty;   /* sampling.cpp:19-28; skipped if ==1            */
  int32_t greedy;             /* !=0: penalty + argmax (text2semantic.cpp:144) */
  int32_t min_tokens_to_keep; /* top_p's third argument (t2s.h:88), default 1 */
} c4s_row_params;

/* Stage bits for c4s_process(): which reference processors to apply, always in
 * the reference order penalty -> temperature -> top_k -> top_p.             */
#define C4S_STAGE_PENALTY 1
#define C4S_STAGE_TEMPERATURE 2
#define C4S_STAGE_TOP_K 4
#define C4S_STAGE_TOP_P 8

/* Debug flags for c4s_set_debug(): force the slow exact paths so that tests
 * can check them on ordinary inputs.                                        */
#define C4S_DEBUG_FORCE_EXACT 1 /* exact sequential sums; radix-select top-k   */
#define C4S_DEBUG_FORCE_BINS 2  /* binned top-p and row-pass draw paths        */
#define C4S_DEBUG_FORCE_REFINE 4 /* no-top-k list rows: exact tail before their list job decides */
#define C4S_DEBUG_SPLIT_PATH 8   /* batches of up to 256 rows: sample through the split kernels
                                    (row, list, general) instead of the fused kernel */
#define C4S_DEBUG_FUSED_PATH 32  /* larger batches: sample through the fused kernel instead of the
                                    split kernels */
#define C4S_DEBUG_FAIL_AFTER_ROW 16 /* split path: fail the list-kernel launch on the host (no kernel
                                    runs or faults), to test recovery of the next call */

/* Device-side error bits reported by c4s_get_status().                     */
#define C4S_DEVERR_HIST_RANGE 1u /* a row's history offsets were out of range */
#define C4S_DEVERR_TIMEOUT 2u    /* a bounded wait on a bulk copy gave up      */
#define C4S_DEVERR_HIST_FULL 8u  /* c4s_decode_step: a row's history window was full
                                    (or its id outside the embedding); the row stopped */
#define C4S_DEVERR_SHARD 4u      /* vocab-sharded merge: a row it cannot decide
                                    exactly (top_k outside [1, 64], or more than
                                    64 of a shard's values tied at the top_k
                                    threshold); the row's id is -1            */

/* Counter slots reported by c4s_get_status() (rows that took each path).    */
#define C4S_CNT_TOPP_EXACT_FALLBACK 0 /* top-p guard band hit: exact re-sum   */
#define C4S_CNT_DRAW_EXACT_FALLBACK 1 /* draw guard band hit: exact re-sum    */
#define C4S_CNT_TOPK_RADIX 2          /* top-k needed the full radix select   */
#define C4S_CNT_TOPP_BINNED 3         /* top-p over more survivors than one warp sorts */
#define C4S_CNT_DRAW_ROWPASS 4        /* draw over more survivors than one warp sorts */
#define C4S_CNT_DEFERRED 5            /* rows the fast kernel left to the general path */
#define C4S_CNT_EXACT_TAIL 6          /* rows without top-k decided after an exact tail sum */
#define C4S_NUM_COUNTERS 8

typedef struct c4s_ctx c4s_ctx;

/* Library ABI version (C4S_ABI_VERSION). */
int c4s_version(void);

/* Human-readable name of a c4s_status. */
const char* c4s_status_string(int status);

/* Create a context on `device` able to process rows of up to `max_vocab`
 * logits. Allocates all device workspace the other calls need. The current
 * device of the calling thread is left unchanged.
 * Replaces: nothing in the reference (its processors allocate per call:
 * sampling.cpp:22,33,45,52).                                                */
int c4s_create(c4s_ctx** out, int32_t max_vocab, int32_t device);

/* As c4s_create, with the workspace sized for batches of up to `max_rows`
 * rows per call (c4s_create = max_rows 4096: about 0.76 GB at max_vocab
 * 8194, most of it candidate lists of 72 KB per row of a 4096-row chunk).
 * Larger batches still run: the split path takes them in chunks of
 * max_rows (rounded up to 32, at most 4096) and the fused and general
 * kernels with at most 2 * max_rows and max_rows CTAs. max_rows 1 (one
 * row per call, as the reference's processors take) needs about 5 MB.
 * Replaces: nothing in the reference.                                      */
int c4s_create_sized(c4s_ctx** out, int32_t max_vocab, int32_t max_rows, int32_t device);
int c4s_destroy(c4s_ctx* ctx);

/* Text of the last error seen by this context ("" if none). */
const char* c4s_last_error(const c4s_ctx* ctx);

/* Set C4S_DEBUG_* flags (0 for production behaviour). */
int c4s_set_debug(c4s_ctx* ctx, int32_t flags);

/* Seed B xorshift64 states: state[b] = (seed ? seed : 0x9E3779B97F4A7C15)
 *                                      + (row_offset + b) * 0x100000001b3.
 * Replaces text2semantic.cpp:109 (single stream = row 0) and :292-295.     */
int c4s_seed_states(uint64_t* d_state, int32_t B, uint64_t seed,
                    int64_t row_offset, void* stream);

/* One sampling step over B rows: for each active row b,
 *   repetition penalty over hist[hist_off[b] .. hist_off[b+1]),
 *   then greedy ? argmax : temperature, top_k, top_p, xorshift64 draw.
 * Replaces the per-row body of text2semantic.cpp:303-331 (and :142-165).
 *   d_logits   fp32 [B, ld], read only; ld >= V (any ld, rows may be unaligned)
 *   d_hist     int32 token history (generated ids, no prompt), CSR by
 *   d_hist_off int64 [B+1]; hist_total = number of ids in d_hist. Ids outside
 *              [0, V) are skipped (sampling.cpp:24). d_hist_off may be NULL:
 *              no history for any row.
 *   d_params   c4s_row_params, per row (stride 1) or broadcast (stride 0)
 *   d_rng      uint64 [B] xorshift64 state, advanced once per sampled row;
 *              greedy and inactive rows leave it unchanged (:304, :144)
 *   d_active   uint8 [B] or NULL (all active); inactive rows get id -1 and
 *              are not touched otherwise
 *   d_out_ids  int32 [B] sampled token ids
 *   d_out_logits  NULL, or fp32 [B, out_ld]: the processed logits of each
 *              active row (what the reference's vector holds before its draw)
 */
int c4s_sample(c4s_ctx* ctx, const float* d_logits, int32_t B, int32_t V,
               int64_t ld, const int32_t* d_hist, const int64_t* d_hist_off,
               int64_t hist_total, const c4s_row_params* d_params,
               int32_t params_stride, uint64_t* d_rng, const uint8_t* d_active,
               int32_t* d_out_ids, float* d_out_logits, int64_t out_ld,
               void* stream);

/* c4s_sample with each row's history given as a window of d_hist:
 * [d_hist_start[b], d_hist_start[b] + d_hist_len[b]) (int64 starts, int32
 * lengths, both [B]; both NULL: no history). Histories that grow in place on
 * the device (c4s_decode_step) are read this way without repacking a CSR
 * array. Same semantics and replacement as c4s_sample.                     */
int c4s_sample_windows(c4s_ctx* ctx, const float* d_logits, int32_t B, int32_t V, int64_t ld,
                       const int32_t* d_hist, const int64_t* d_hist_start, const int32_t* d_hist_len,
                       int64_t hist_total, const c4s_row_params* d_params, int32_t params_stride,
                       uint64_t* d_rng, const uint8_t* d_active, int32_t* d_out_ids, float* d_out_logits,
                       int64_t out_ld, void* stream);

/* The bookkeeping of one decode step after sampling, on the device
 * (text2semantic.cpp:167-178 single stream, :333-351 batched), for B rows:
 *   an active row (d_active NULL: every row) whose id is stop_token becomes
 *   inactive and counts in *d_done_count; any other active row appends its id
 *   to its history window (d_hist at d_hist_start[b], length d_hist_len[b] <
 *   hist_cap, advanced) and, with d_latents, the hidden state d_cur[b] that
 *   predicted it to latents [B][hist_cap][D]; a full window stops the row
 *   (C4S_DEVERR_HIST_FULL). Then every row's next input embedding:
 *   d_next_emb[b] = d_emb[tok] + d_pos_emb (bf16 adds rounded to nearest
 *   even; d_pos_emb is the position row for this step), tok = the appended
 *   id, 0 for rows that did not append (as the reference embeds them).
 * bf16 tensors are uint16_t bit patterns, rows of D contiguous elements;
 * d_cur may be the d_next_emb buffer itself.                               */
int c4s_decode_step(c4s_ctx* ctx, const int32_t* d_ids, int32_t B, uint8_t* d_active, int32_t stop_token,
                    int32_t* d_hist, const int64_t* d_hist_start, int32_t* d_hist_len, int32_t hist_cap,
                    const uint16_t* d_emb, int32_t n_emb, const uint16_t* d_pos_emb, int32_t D,
                    uint16_t* d_next_emb, const uint16_t* d_cur, uint16_t* d_latents,
                    uint32_t* d_done_count, void* stream);

/* ------------------------------------------------------------------------
 * Quantized decode GEMVs of the T2S GPT-2. The reference's default build
 * (apps/c4tts_cli.cpp:300-306, C4TTS_QUANT=8) quantizes each projection weight
 * once (gpt2.cpp:52-60: the (out, in) weight, mx::quantize, group 64) and runs
 * the decode projections as quantized_matmul(x, w_q, scales, biases,
 * transpose=true) + bias (gpt2.cpp:61-63). Affine scheme, per group of
 * `group` consecutive weights of a row: scale = (max - min) / (2^bits - 1),
 * bias = min, q = round((w - bias) / scale) (half to even); w ~= scale q + bias;
 * codes packed little-end-first in 32-bit words.
 *   c4s_quantize_affine: w fp32 [N, K] -> d_q uint32 [N, K * bits / 32],
 *                        scales / biases fp32 [N, K / group];
 *   c4s_qgemv:           y fp32 [B, N] = x fp32 [B, K] dequant(q)^T + bias_out
 *                        (bias_out fp32 [N] or NULL), fp32 accumulation; built
 *                        for decode batches (weight-bandwidth bound).
 * bits 4 or 8; group 32, 64 or 128 dividing K; K <= 8192 for the GEMV.     */
int c4s_quantize_affine(c4s_ctx* ctx, const float* d_w, int32_t N, int32_t K, int32_t group, int32_t bits,
                        uint32_t* d_q, float* d_scales, float* d_biases, void* stream);
int c4s_qgemv(c4s_ctx* ctx, const float* d_x, int32_t B, int32_t K, const uint32_t* d_q, const float* d_scales,
              const float* d_biases, int32_t N, int32_t group, int32_t bits, const float* d_bias_out, float* d_y,
              void* stream);

/* Apply the processors selected by `stages` (C4S_STAGE_* bits) in place to B
 * rows of d_logits, in the reference order, ignoring params.greedy.
 * Replaces the in-place processors of sampling.cpp:14-71 / t2s.h:83-88:
 *   repetition_penalty (sampling.cpp:19), temperature (:14), top_k (:30),
 *   top_p (:42).                                                           */
int c4s_process(c4s_ctx* ctx, float* d_logits, int32_t B, int32_t V,
                int64_t ld, const int32_t* d_hist, const int64_t* d_hist_off,
                int64_t hist_total, const c4s_row_params* d_params,
                int32_t params_stride, int32_t stages, void* stream);

/* First index of the row maximum for B rows (std::max_element semantics).
 * Replaces argmax, sampling.cpp:73-76 / t2s.h:89.                          */
int c4s_argmax(c4s_ctx* ctx, const float* d_logits, int32_t B, int32_t V,
               int64_t ld, int32_t* d_out_ids, void* stream);

/* Synchronise `stream`, then report (and optionally clear) the device error
 * bits (C4S_DEVERR_*) and path counters (C4S_CNT_*; may be NULL).
 * Returns C4S_ERR_DEVICE / C4S_ERR_TIMEOUT if an error bit is set.          */
int c4s_get_status(c4s_ctx* ctx, uint32_t* dev_errors,
                   uint64_t* counters /* [C4S_NUM_COUNTERS] or NULL */,
                   int32_t reset, void* stream);

/* Measurement only; no counterpart in the reference. While enabled, every
 * c4s_sample call that takes the fast path records CUDA events on its stream
 * around its kernels: the fused kernel (one launch per call), or, on the
 * split path (C4S_DEBUG_SPLIT_PATH), per chunk of 4096 rows the order
 * pre-pass (rows by cost class; only when a chunk has more rows than the row
 * kernel has CTAs and per-row parameters), the row, list and general kernels.
 * c4s_kernel_times waits for them and returns the summed device times in
 * milliseconds and the number of launches of each kernel in ms[5] /
 * launches[5], in the order order, row, list, general, fused; reset forgets
 * the recorded calls. Not for use while a stream is being captured.         */
#define C4S_NUM_KERNEL_TIMERS 5
int c4s_kernel_timing(c4s_ctx* ctx, int32_t enable);
int c4s_kernel_times(c4s_ctx* ctx, double* ms, int64_t* launches, int32_t reset);

/* c4s_sample without a context, for callers that must not allocate device
 * memory at all. No counterpart in the reference (whose sampling stage has no
 * device state); it exists so that a caller can sample before, or without,
 * creating a context.
 *   - Same arguments and results as c4s_sample (no processed logits); it runs
 *     the general kernel on at most 16 CTAs.
 *   - Scratch is a file-scope device array of C4S_STATIC_MAX_VOCAB * 16 keys
 *     (2 MiB): V above C4S_STATIC_MAX_VOCAB returns C4S_ERR_CAPACITY.
 *   - Nothing is allocated, by this call or the library. The first call on a
 *     device (the calling thread's current device) looks up the array's device
 *     address and sets the kernel's shared-memory attribute; make that first
 *     call before any stream capture.
 *   - All calls on a device share the array: calls that overlap in time (on
 *     different streams or threads) race and must be serialised by the caller.
 *   - The device error flags and path counters that the kernel writes are
 *     cleared (stream-ordered) at the start of every call; they are not
 *     reported: validate history offsets before calling. A row whose bulk
 *     copy was not seen to complete within the kernel's bounded wait (about
 *     2 s) gets id -1, as do the later rows of its CTA.                     */
#define C4S_STATIC_MAX_VOCAB 16384
int c4s_sample_static(const float* d_logits, int32_t B, int32_t V, int64_t ld,
                      const int32_t* d_hist, const int64_t* d_hist_off,
                      int64_t hist_total, const c4s_row_params* d_params,
                      int32_t params_stride, uint64_t* d_rng,
                      const uint8_t* d_active, int32_t* d_out_ids, void* stream);

/* ------------------------------------------------------------------------
 * LM head of the T2S decoder on tcgen05 tensor cores. The reference computes
 * per step (text2semantic.cpp:118-121, batched :283-286)
 *     logits = linear(layer_norm(h, final_norm.weight, final_norm.bias),
 *                     semantic_head.weight, semantic_head.bias)
 * (nn.cpp:73-83: biased variance, (x - mean) / sqrt(var + eps); nn.cpp:11-16:
 * y W^T + b with W = (out, in)) and copies the logits to the host.
 *   d_hidden  bf16 [B, ld_hidden]          d_gamma, d_beta  fp32 [d] or NULL (1, 0)
 *   d_weight  bf16 [N, ld_weight] (out x in, as the checkpoint stores it)
 *   d_bias    fp32 [N] or NULL             d_logits  fp32 [B, ld_logits] (output)
 *   d_norm    bf16 [B, d]: caller-owned workspace for the normalised states,
 *             the GEMM's A operand; NULL skips the LayerNorm (logits =
 *             hidden W^T + b, nn.cpp:11-16 alone).
 * The GEMM accumulates in fp32 (bf16 products are exact in fp32). d is a
 * multiple of 64 (of 128 with the LayerNorm), at most 8192; weight rows (and
 * hidden rows without the LayerNorm) 16-byte aligned. bf16 values are passed
 * as uint16_t bit patterns.                                                  */
int c4s_head_logits(c4s_ctx* ctx, const uint16_t* d_hidden, int32_t B, int32_t d, int64_t ld_hidden,
                    const float* d_gamma, const float* d_beta, float eps, const uint16_t* d_weight, int32_t N,
                    int64_t ld_weight, const float* d_bias, uint16_t* d_norm, float* d_logits, int64_t ld_logits,
                    void* stream);

/* c4s_head_logits, then c4s_sample on the logits (same semantics and
 * arguments; N is the vocabulary): one decode step's head and sampling with
 * no host round trip. Replaces text2semantic.cpp:134-165 (single stream) and
 * :296-331 (batched) after the GPT-2 forward pass.                         */
int c4s_head_sample(c4s_ctx* ctx, const uint16_t* d_hidden, int32_t B, int32_t d, int64_t ld_hidden,
                    const float* d_gamma, const float* d_beta, float eps, const uint16_t* d_weight, int32_t N,
                    int64_t ld_weight, const float* d_bias, uint16_t* d_norm, float* d_logits, int64_t ld_logits,
                    const int32_t* d_hist, const int64_t* d_hist_off, int64_t hist_total,
                    const c4s_row_params* d_params, int32_t params_stride, uint64_t* d_rng,
                    const uint8_t* d_active, int32_t* d_out_ids, void* stream);

/* Test hook, no counterpart in the reference: d_out[i] = x[i] / d computed by
 * the kernels' inline division (a Markstein-corrected reciprocal product with
 * a proof check, else the IEEE division), so that tests can compare it bit
 * for bit with IEEE round-to-nearest division (sampling.cpp:16, :26).      */
int c4s_test_div_rn(const float* d_x, float d, float* d_out, int64_t n, void* stream);

/* ------------------------------------------------------------------------
 * Vocab-sharded sampling: the vocabulary of every row is split into
 * contiguous shards (one per GPU), and no GPU holds a whole row. One step is
 *
 *   c4s_shard_candidates  on every shard: penalty (history ids inside the
 *                         shard), temperature, the shard's 64 largest values;
 *   all-gather            of the [B][64] candidate blocks of all shards
 *                         (ncclAllGather, 512 B per row and shard);
 *   c4s_merge_candidates  on every GPU: greedy argmax, or top_k, top_p and the
 *                         xorshift64 draw over the gathered candidates.
 *
 * Every GPU gets the same ids and advances the same xorshift64 states. For
 * sampled rows the result equals c4s_sample on the whole row (the reference's
 * text2semantic.cpp:303-331) when 1 <= top_k <= 64; other sampled rows are
 * refused per row (id -1, C4S_DEVERR_SHARD). The reference has no vocab
 * sharding; these two calls together replace the same per-row body as
 * c4s_sample (text2semantic.cpp:303-331).                                  */
#define C4S_SHARD_CANDIDATES 64
#define C4S_MAX_SHARDS 16
#define C4S_CAND_TIES 0x80000000u /* set in the last candidate's index when the
                                     shard has more values equal to its 64th */
typedef struct c4s_candidate {
  float value;    /* penalised (and, for sampled rows, tempered) logit        */
  int32_t index;  /* global vocabulary index; bit 31 = C4S_CAND_TIES         */
} c4s_candidate;

/* Candidates of one shard for B rows.
 *   d_logits      fp32 [B, ld]: this shard's V_shard columns of every row
 *                 (ld >= V_shard; 4-byte aligned rows)
 *   vocab_offset  global index of the shard's first column; the shard covers
 *                 [vocab_offset, vocab_offset + V_shard) of [0, V)
 *   d_hist..params_stride, d_active   as for c4s_sample (history ids are
 *                 global; each shard penalises the ones it holds)
 *   d_cand        c4s_candidate [B][C4S_SHARD_CANDIDATES], largest value
 *                 first, ties by ascending index; inactive rows are skipped.
 * 64 <= V_shard <= 32768.                                                   */
int c4s_shard_candidates(c4s_ctx* ctx, const float* d_logits, int32_t B,
                         int32_t V_shard, int64_t ld, int32_t vocab_offset,
                         int32_t V, const int32_t* d_hist,
                         const int64_t* d_hist_off, int64_t hist_total,
                         const c4s_row_params* d_params, int32_t params_stride,
                         const uint8_t* d_active, c4s_candidate* d_cand,
                         void* stream);

/* Candidates of every shard of whole rows held by one GPU, in one launch:
 * d_logits fp32 [B, ld] (ld >= V) holds whole rows; shard s is the column
 * block starting at s*(V/G) + min(s, V%G), of width V/G (+1 for s < V%G),
 * G = num_shards (1..C4S_MAX_SHARDS, every shard 64..32768 wide); shard s's
 * [B][64] block is written at d_cand + s * shard_stride (>= B * 64), the
 * layout c4s_merge_candidates reads. With c4s_merge_candidates this is the
 * single-GPU form of the vocab-sharded step, and samples rows wider than
 * c4s_sample's 32768 columns (for 1 <= top_k <= 64). Replaces the same
 * per-row body of text2semantic.cpp:303-331 as c4s_sample.                 */
int c4s_shard_candidates_split(c4s_ctx* ctx, const float* d_logits, int32_t B,
                               int32_t V, int64_t ld, int32_t num_shards,
                               const int32_t* d_hist, const int64_t* d_hist_off,
                               int64_t hist_total, const c4s_row_params* d_params,
                               int32_t params_stride, const uint8_t* d_active,
                               c4s_candidate* d_cand, int64_t shard_stride,
                               void* stream);

/* The candidates of one GPU's vocabulary shard [vocab_offset, vocab_offset +
 * V_shard) of [0, V) (arguments as c4s_shard_candidates), computed as
 * `num_sub` contiguous sub-shards of the shard's columns (split as
 * c4s_shard_candidates_split splits whole rows; every sub-shard 64..32768
 * wide): sub-shard s's [B][64] block at d_cand + s * shard_stride. A rank
 * whose shard is wide (32768 columns of a 65536 vocabulary on two GPUs)
 * keeps several CTAs per SM this way; the gathered blocks of all ranks,
 * rank-major, are in vocabulary order for c4s_merge_candidates.
 * Replaces the same per-row body of text2semantic.cpp:303-331.             */
int c4s_shard_candidates_sub(c4s_ctx* ctx, const float* d_logits, int32_t B,
                             int32_t V_shard, int64_t ld, int32_t vocab_offset,
                             int32_t V, int32_t num_sub, const int32_t* d_hist,
                             const int64_t* d_hist_off, int64_t hist_total,
                             const c4s_row_params* d_params, int32_t params_stride,
                             const uint8_t* d_active, c4s_candidate* d_cand,
                             int64_t shard_stride, void* stream);

/* Token ids from the candidates of `num_shards` shards (1..C4S_MAX_SHARDS),
 * shard s's block at d_cand + s * shard_stride (shard_stride >= B * 64, in
 * candidates: the layout of an all-gather of the [B][64] blocks, shards in
 * vocabulary order). d_rng, d_active and d_out_ids as for c4s_sample.        */
int c4s_merge_candidates(c4s_ctx* ctx, const c4s_candidate* d_cand,
                         int32_t num_shards, int64_t shard_stride, int32_t B,
                         int32_t V, const c4s_row_params* d_params,
                         int32_t params_stride, uint64_t* d_rng,
                         const uint8_t* d_active, int32_t* d_out_ids,
                         void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* C4S_SAMPLING_H_ */
