"""Device-resident batched T2S decode driver.

The reference's Text2Semantic::generate_batch (src/t2s/text2semantic.cpp:196-373
of the reference) runs, per step, the head on the GPT-2 output, copies the
logits to the host, samples every unfinished stream in scalar C++, appends the
ids to per-stream histories, marks streams that drew the stop token as done
and embeds the new tokens for the next forward pass. DecodeLoop keeps all of
that on the device:

    head_logits      LayerNorm + LM head on the tensor cores (c4s_head_logits)
    sample_windows   penalty / temperature / top-k / top-p / xorshift64 draw of
                     every active row, histories read in place (c4s_sample_windows)
    decode_step      stop-token check, history and latent append, next
                     embeddings (c4s_decode_step)

The GPT-2 forward pass itself (the KV-cached transformer) is the caller's: it
is a function next_embeddings -> hidden states handed to run(). Nothing crosses
to the host per step except, every `poll_every` steps, the count of finished
streams. Rows that finish keep their RNG state and history; once every row is
done the loop stops (at most poll_every - 1 steps later, steps in which no row
is active and nothing changes).
"""
from __future__ import annotations

import numpy as np

from . import workloads


class DecodeLoop:
    """Per-stream state of a batched decode on one GPU.

    ctx           SamplingContext (its device and stream)
    head          dict of CUDA tensors: weight bf16 [V, d] (int16 bits), bias
                  fp32 [V] or None, gamma / beta fp32 [d] (final_norm) or None
    emb           bf16 [V_emb, d] semantic_embedding.weight
    pos_emb       bf16 [max_pos, d] semantic_position_embedding.weight
                  (row step + 1 embeds the token drawn at `step`, the BOS
                  holding row 0, text2semantic.cpp:172-177)
    params        workloads.ROW_PARAMS_DTYPE [B] (or one struct)
    seed          xorshift64 seeding of text2semantic.cpp:292-295
    """

    def __init__(self, ctx, B: int, head: dict, emb, pos_emb, params, seed: int = 1234,
                 max_new_tokens: int = 1000, stop_token: int = workloads.STOP_TOKEN,
                 keep_latents: bool = False, eps: float = 1e-5):
        import torch
        self.ctx, self.B, self.head = ctx, B, head
        self.emb, self.pos_emb = emb, pos_emb
        self.cap, self.stop, self.eps = max_new_tokens, stop_token, eps
        dev = emb.device
        self.V = head["weight"].shape[0]
        self.d = head["weight"].shape[1]
        if emb.shape[1] != self.d or pos_emb.shape[1] != self.d:
            raise ValueError("embedding widths must match the head's input width")
        if pos_emb.shape[0] < max_new_tokens + 1:
            raise ValueError("position table shorter than max_new_tokens + 1 rows")
        p = np.asarray(params, dtype=workloads.ROW_PARAMS_DTYPE)
        self.params_stride = 0 if p.shape == () or p.size == 1 else 1
        from .sampling import params_tensor
        self.params = params_tensor(p.reshape(-1), dev)
        self.hist = torch.zeros(B * max(1, max_new_tokens), dtype=torch.int32, device=dev)
        self.hist_start = torch.arange(B, dtype=torch.int64, device=dev) * max(1, max_new_tokens)
        self.hist_len = torch.zeros(B, dtype=torch.int32, device=dev)
        self.active = torch.ones(B, dtype=torch.uint8, device=dev)
        self.rng = ctx.seed_states(B, seed)
        self.ids = torch.empty(B, dtype=torch.int32, device=dev)
        self.logits = torch.empty((B, self.V), dtype=torch.float32, device=dev)
        self.norm = torch.empty((B, self.d), dtype=torch.int16, device=dev)
        self.next_emb = torch.empty((B, self.d), dtype=torch.int16, device=dev)
        self.done = torch.zeros(1, dtype=torch.int32, device=dev)
        self.latents = (torch.zeros((B, max(1, max_new_tokens), self.d), dtype=torch.int16, device=dev)
                        if keep_latents else None)
        self.steps = 0

    def step(self, hidden):
        """One decode step on hidden states bf16 [B, d] (the forward pass's
        last position): head, sampling, bookkeeping. Returns next embeddings."""
        s = self.steps
        if s >= self.cap:
            raise RuntimeError("max_new_tokens reached")
        h = self.head
        self.ctx.head_logits(hidden, h["weight"], h.get("bias"), h.get("gamma"), h.get("beta"), eps=self.eps,
                             norm_out=self.norm, logits_out=self.logits)
        self.ctx.sample_windows(self.logits, self.hist, self.hist_start, self.hist_len, self.params, self.rng,
                                active=self.active, out_ids=self.ids, params_stride=self.params_stride)
        self.ctx.decode_step(self.ids, self.active, self.stop, self.hist, self.hist_start, self.hist_len, self.cap,
                             self.emb, self.pos_emb[s + 1], self.next_emb, self.done,
                             cur=hidden if self.latents is not None else None, latents=self.latents)
        self.steps += 1
        return self.next_emb

    def finished(self) -> int:
        """Streams that drew the stop token (one device-to-host read)."""
        return int(self.done.item())

    def run(self, forward, hidden, poll_every: int = 8):
        """Decode until every stream is done or max_new_tokens steps ran;
        forward(next_embeddings, step) -> hidden states of the next step."""
        while self.steps < self.cap:
            nxt = self.step(hidden)
            if self.steps % poll_every == 0 and self.finished() >= self.B:
                break
            if self.steps < self.cap:
                hidden = forward(nxt, self.steps - 1)
        return self.results()

    def results(self):
        """Per stream: generated ids (int32 numpy) and, if kept, latents
        (bf16 bits [n, d]) -- the reference's Generation{codes, latent}."""
        lens = self.hist_len.cpu().numpy()
        hist = self.hist.cpu().numpy().reshape(self.B, -1)
        out = []
        lat = None if self.latents is None else self.latents.cpu().numpy().view(np.uint16)
        for b in range(self.B):
            n = int(lens[b])
            out.append((hist[b, :n].copy(), None if lat is None else lat[b, :n].copy()))
        return out
