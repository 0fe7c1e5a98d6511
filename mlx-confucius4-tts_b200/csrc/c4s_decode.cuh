// c4s_decode.cuh -- the bookkeeping of one T2S decode step, on the device.
//
// After the sampling step the reference (text2semantic.cpp:167-178 single
// stream, :333-351 batched) does, per stream b that is still generating:
//   tok == stop token (8193): the stream is done (its RNG has already
//     advanced); nothing is appended;
//   else: tok is appended to the stream's generated ids (the repetition
//     penalty's history) and the hidden state that predicted it to its
//     latents (the S2A stage's input);
// then embeds every stream's token for the next forward pass:
//   next[b] = semantic_embedding[tok_b] + semantic_position_embedding[step + 1],
// with token 0 for streams that are done (their entry of tok_arr stays 0).
// decode_step_kernel does all of it for a batch in one launch, so the token
// ids, histories, done flags and next embeddings never cross to the host.
// Histories live in per-row windows [start[b], start[b] + len[b]) of capacity
// cap (c4s_sample_windows reads them in place); the done count lets the host
// poll for the end of the loop every few steps instead of every step.
#pragma once

namespace c4s {

struct DecodeArgs {
  const int* ids;                 // [B] sampled ids (-1: row was inactive)
  int B;
  unsigned char* active;          // [B] or null (every row generating)
  int stop;
  int* hist;                      // generated ids, row b's window at hist_start[b]
  const long long* hist_start;    // [B]
  int* hist_len;                  // [B], advanced here
  int hist_cap;
  const unsigned short* emb;      // bf16 [n_emb, D]  semantic_embedding.weight
  int n_emb;
  const unsigned short* pos_emb;  // bf16 row `pos` of semantic_position_embedding.weight [*, D]
  int D;
  unsigned short* next_emb;       // bf16 [B, D]
  const unsigned short* cur;      // bf16 [B, D] hidden state that predicted ids (null: no latents)
  unsigned short* latents;        // bf16 [B, hist_cap, D] or null
  unsigned* done_count;           // streams that finished (incremented here)
  unsigned* errflags;
};

__device__ __forceinline__ unsigned short bf16_add(unsigned short a, unsigned short b) {
  const float s = __uint_as_float((unsigned)a << 16) + __uint_as_float((unsigned)b << 16);
  const unsigned u = __float_as_uint(s);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (unsigned short)((u >> 16) | 0x40u);   // NaN stays NaN
  return (unsigned short)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);                   // nearest even
}

constexpr int DEC_NT = 128;
__global__ void __launch_bounds__(DEC_NT) decode_step_kernel(DecodeArgs g) {
  __shared__ int tok_e, slot;
  grid_dep_wait();                                 // the sampling step's ids (and everything before it)
  grid_dep_launch();
  const int b = blockIdx.x;
  if (threadIdx.x == 0) {
    int te = 0, sl = -1;
    if (g.active == nullptr || g.active[b]) {
      const int tok = g.ids[b];
      if (tok == g.stop) {
        if (g.active) g.active[b] = 0;
        atomicAdd(g.done_count, 1u);
      } else {
        const int len = g.hist_len[b];
        if (len < 0 || len >= g.hist_cap || tok < 0 || tok >= g.n_emb) {
          // a full history window (or an id the embedding cannot take): the
          // row stops generating and the flag reports it
          atomicOr(g.errflags, C4S_DEVERR_HIST_FULL);
          if (g.active) g.active[b] = 0;
          atomicAdd(g.done_count, 1u);
        } else {
          g.hist[g.hist_start[b] + len] = tok;
          g.hist_len[b] = len + 1;
          te = tok;
          sl = len;
        }
      }
    }
    tok_e = te;
    slot = sl;
  }
  __syncthreads();
  // the latent first: cur may be the next_emb buffer itself (a caller that
  // feeds the embeddings back), and each CTA touches only its own row
  if (slot >= 0 && g.latents && g.cur) {
    const unsigned short* c = g.cur + (long long)b * g.D;
    unsigned short* l = g.latents + ((long long)b * g.hist_cap + slot) * g.D;
    for (int i = threadIdx.x; i < g.D; i += DEC_NT) l[i] = c[i];
  }
  __syncthreads();
  const unsigned short* er = g.emb + (long long)tok_e * g.D;
  unsigned short* o = g.next_emb + (long long)b * g.D;
  for (int i = threadIdx.x; i < g.D; i += DEC_NT) o[i] = bf16_add(er[i], g.pos_emb[i]);
}

}  // namespace c4s
