"""Seeded synthetic inputs for the T2S sampling stage.

There is no public dataset for this path: the reference measures nothing but
the per-step sampling time of its own decode loop. These generators stand in
for real semantic-head logits with the shapes and value distributions the
benchmark configurations name (logits ~N(0, 3^2) over the 8194-token semantic
vocabulary, uniform token histories, the reference's sampling defaults from
include/c4tts/pipeline.h:26-37 of the reference).

Everything is numpy on the host; callers upload what they need.
"""
from __future__ import annotations

import dataclasses

import numpy as np

SEMANTIC_VOCAB = 8194          # t2s semantic head width (8192 codes + BOS + EOS)
STOP_TOKEN = 8193              # text2semantic.cpp:167 (stop_semantic_token)
GOLDEN_STATE = 0x9E3779B97F4A7C15   # text2semantic.cpp:109 (seed 0)
ROW_STRIDE = 0x100000001B3          # text2semantic.cpp:294

# numpy structured dtype with the exact layout of c4s_row_params.
ROW_PARAMS_DTYPE = np.dtype([
    ("temperature", "<f4"),
    ("top_k", "<i4"),
    ("top_p", "<f4"),
    ("repetition_penalty", "<f4"),
    ("greedy", "<i4"),
    ("min_tokens_to_keep", "<i4"),
])
assert ROW_PARAMS_DTYPE.itemsize == 24


def seed_states(B: int, seed: int, row_offset: int = 0) -> np.ndarray:
    """xorshift64 states of rows [row_offset, row_offset + B) (text2semantic.cpp:292-295)."""
    base = seed if seed else GOLDEN_STATE
    b = np.arange(row_offset, row_offset + B, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return (np.uint64(base) + b * np.uint64(ROW_STRIDE)).astype(np.uint64)


def make_params(B: int, temperature=0.8, top_k=30, top_p=0.8,
                repetition_penalty=10.0, greedy=0, min_tokens_to_keep=1) -> np.ndarray:
    """Per-row params array; scalars broadcast, arrays are taken per row."""
    p = np.zeros(B, dtype=ROW_PARAMS_DTYPE)
    p["temperature"] = temperature
    p["top_k"] = top_k
    p["top_p"] = top_p
    p["repetition_penalty"] = repetition_penalty
    p["greedy"] = greedy
    p["min_tokens_to_keep"] = min_tokens_to_keep
    return p


@dataclasses.dataclass
class Batch:
    """One sampling step's inputs for B rows (host arrays)."""
    logits: np.ndarray      # float32 [B, ld]
    V: int
    hist: np.ndarray        # int32 [total]
    hist_off: np.ndarray    # int64 [B + 1]
    params: np.ndarray      # ROW_PARAMS_DTYPE [B]
    rng: np.ndarray         # uint64 [B]

    @property
    def B(self) -> int:
        return self.logits.shape[0]

    @property
    def ld(self) -> int:
        return self.logits.shape[1]


def normal_logits(rng: np.random.Generator, B: int, V: int, sigma=3.0,
                  spikes=0, spike=12.0, ld: int | None = None) -> np.ndarray:
    """float32 [B, ld] ~N(0, sigma^2) with `spikes` +spike bumps per row."""
    ld = V if ld is None else ld
    x = np.zeros((B, ld), dtype=np.float32)
    x[:, :V] = rng.normal(0.0, sigma, size=(B, V)).astype(np.float32)
    if spikes:
        pos = rng.integers(0, V, size=(B, spikes))
        rows = np.repeat(np.arange(B), spikes)
        np.add.at(x, (rows, pos.ravel()), np.float32(spike))
    return x


def csr_history(rng: np.random.Generator, lengths: np.ndarray, hi=8192):
    """CSR token history with the given per-row lengths, ids uniform in [0, hi)."""
    off = np.zeros(len(lengths) + 1, dtype=np.int64)
    np.cumsum(lengths, out=off[1:])
    hist = rng.integers(0, hi, size=int(off[-1]), dtype=np.int64).astype(np.int32)
    return hist, off


def config0(seed: int = 0, V: int = SEMANTIC_VOCAB, greedy: bool = False) -> Batch:
    """c0: single stream, history 256, pen 10 / T 0.8 / k 30 / p 0.8, state seed 0."""
    g = np.random.default_rng(1000 + seed)
    logits = normal_logits(g, 1, V, spikes=5)
    hist, off = csr_history(g, np.array([256]))
    return Batch(logits, V, hist, off, make_params(1, greedy=int(greedy)),
                 seed_states(1, 0))


def config1(seed: int = 1, B: int = 64, V: int = SEMANTIC_VOCAB) -> Batch:
    """c1: B=64 streams, row-varying spikes, history 1024/row, keys from seed 1."""
    g = np.random.default_rng(2000 + seed)
    logits = normal_logits(g, B, V, spikes=5)
    hist, off = csr_history(g, np.full(B, 1024))
    return Batch(logits, V, hist, off, make_params(B), seed_states(B, 1))


def config2(seed: int = 2, B: int = 4096, V: int = SEMANTIC_VOCAB,
            row_offset: int = 0, ld: int | None = None) -> Batch:
    """c2: server-scale heterogeneous batch (ragged history U[0,2048], per-row params)."""
    g = np.random.default_rng([3000 + seed, row_offset])
    logits = normal_logits(g, B, V, ld=ld)
    hist, off = csr_history(g, g.integers(0, 2049, size=B))
    params = make_params(
        B,
        temperature=g.uniform(0.5, 1.2, size=B).astype(np.float32),
        top_k=g.choice(np.array([0, 20, 50, 200], dtype=np.int32), size=B),
        top_p=g.uniform(0.6, 1.0, size=B).astype(np.float32),
        repetition_penalty=g.uniform(1.0, 10.0, size=B).astype(np.float32),
    )
    return Batch(logits, V, hist, off, params, seed_states(B, seed, row_offset))


VOCAB_SHARDED_V = 65536       # config 4: 8 contiguous shards of 8192


def config4(seed: int = 4, B: int = 512, V: int = VOCAB_SHARDED_V, top_k: int = 50,
            top_p: float = 0.9) -> Batch:
    """c4: vocab-sharded stress batch -- B=512 rows of V=65536 ~N(0, 3^2),
    history 1024/row with ids uniform over the whole vocabulary, global
    top_k 50 / top_p 0.9 with the reference's other defaults (T 0.8,
    penalty 10), per-row states from seed `seed`."""
    g = np.random.default_rng(5000 + seed)
    logits = normal_logits(g, B, V)
    hist, off = csr_history(g, np.full(B, 1024), hi=V)
    return Batch(logits, V, hist, off, make_params(B, top_k=top_k, top_p=top_p),
                 seed_states(B, seed))


HEAD_DIM = 1280              # GPT-2 hidden size of the T2S model (config 3)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round to nearest even."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def bf16_float(b: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32 (exact)."""
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


@dataclasses.dataclass
class HeadBatch:
    """Config 3 inputs: decoder hidden states and the LM head, bf16 as uint16."""
    hidden: np.ndarray      # uint16 (bf16) [B, d]
    gamma: np.ndarray       # float32 [d]   final_norm.weight
    beta: np.ndarray        # float32 [d]   final_norm.bias
    weight: np.ndarray      # uint16 (bf16) [N, d]  semantic_head.weight (out x in)
    bias: np.ndarray        # float32 [N]   semantic_head.bias
    hist: np.ndarray
    hist_off: np.ndarray
    params: np.ndarray
    rng: np.ndarray

    @property
    def B(self) -> int:
        return self.hidden.shape[0]

    @property
    def N(self) -> int:
        return self.weight.shape[0]


def config3(seed: int = 3, B: int = 256, d: int = HEAD_DIM, N: int = SEMANTIC_VOCAB,
            hist_len: int = 512) -> HeadBatch:
    """c3: fused LM head + sampling -- hidden states bf16 ~N(0, 1) [B, d], head
    weight bf16 ~N(0, 0.02^2) [N, d], LayerNorm affine and head bias near
    their initial values (gamma 1 + N(0, 0.05^2), beta and bias N(0, 0.02^2)),
    history 512 per row, config-0 sampling parameters, states from `seed`."""
    g = np.random.default_rng(4000 + seed)
    hidden = bf16_bits(g.normal(0.0, 1.0, size=(B, d)).astype(np.float32))
    weight = bf16_bits(g.normal(0.0, 0.02, size=(N, d)).astype(np.float32))
    gamma = (1.0 + g.normal(0.0, 0.05, size=d)).astype(np.float32)
    beta = g.normal(0.0, 0.02, size=d).astype(np.float32)
    bias = g.normal(0.0, 0.02, size=N).astype(np.float32)
    hist, off = csr_history(g, np.full(B, hist_len), hi=min(N, 8192))
    return HeadBatch(hidden, gamma, beta, weight, bias, hist, off, make_params(B), seed_states(B, seed))


def head_flops(B: int, d: int, N: int) -> int:
    """Multiply-adds of the head GEMM counted as 2 flops."""
    return 2 * B * d * N


def append_history(hist: np.ndarray, off: np.ndarray, toks: np.ndarray,
                   active: np.ndarray | None = None):
    """Append one token per (active) row to a CSR history (text2semantic.cpp:334)."""
    B = len(off) - 1
    lens = np.diff(off)
    add = np.ones(B, dtype=np.int64) if active is None else active.astype(np.int64)
    new_off = np.zeros(B + 1, dtype=np.int64)
    np.cumsum(lens + add, out=new_off[1:])
    new_hist = np.empty(int(new_off[-1]), dtype=np.int32)
    for b in range(B):
        n = lens[b]
        new_hist[new_off[b]:new_off[b] + n] = hist[off[b]:off[b + 1]]
        if add[b]:
            new_hist[new_off[b] + n] = toks[b]
    return new_hist, new_off


def algorithmic_bytes(V: int, hist_off: np.ndarray, B: int) -> int:
    """Bytes one sampling step must move per batch: 4V logits + 4H history
    + 8 CSR offset + 24 params + 16 RNG read/write + 4 id, per row."""
    H = int(hist_off[-1] - hist_off[0])
    return B * (4 * V + 8 + 24 + 16 + 4) + 4 * H
