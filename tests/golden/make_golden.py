#!/usr/bin/env python3
"""Regenerate the golden fixtures under tests/golden/.

Needs the reference tree ($C4S_REFERENCE, else BASELINE.json's
reference_path) and is run by hand, never by the tests. It writes two kinds of fixtures:

  hf/sampling/*.npy   The reference's own HuggingFace goldens: this script
                      imports the reference's tools/dump_golden.py and calls
                      its dump_sampling() (dump_golden.py:807-825; vocab 64,
                      seed 51, T 0.8, penalty 1.3, k 10, p 0.9), exactly what
                      the reference's tests/test_sampling.cpp consumes.
  ref_*.npz           Outputs of the reference's unmodified
                      src/t2s/sampling.cpp, compiled from source into
                      oracle/_ref/libc4s_ref.so (make -C oracle ref), on seeded
                      synthetic inputs, plus the restated draw for sampled ids.

Usage:  python tests/golden/make_golden.py
"""
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _reference_tree():
    path = os.environ.get("C4S_REFERENCE")
    if not path:
        import json
        with open(os.path.join(REPO, "BASELINE.json")) as f:
            path = json.load(f).get("reference_path")
    if not path or not os.path.isdir(path):
        sys.exit("make_golden.py needs the reference tree: set C4S_REFERENCE")
    return path


REF = _reference_tree()
sys.path.insert(0, os.path.join(REPO, "oracle"))
import oracle as orc  # noqa: E402

spec = importlib.util.spec_from_file_location(
    "c4s_workloads", os.path.join(REPO, "mlx-confucius4-tts_b200", "workloads.py"))
wl = importlib.util.module_from_spec(spec)
sys.modules["c4s_workloads"] = wl
spec.loader.exec_module(wl)


def hf_goldens():
    sys.path.insert(0, os.path.join(REF, "tools"))
    import dump_golden  # the reference's golden dumper
    dump_golden.dump_sampling(os.path.join(HERE, "hf"))


def proc_cases():
    """Single-row processor cases through the reference's own functions."""
    g = np.random.default_rng(51)
    rows, specs = [], []

    def add(x, hist, T, k, p, pen, min_keep=1):
        rows.append(x.astype(np.float32))
        specs.append((len(x), T, k, p, pen, min_keep, hist.astype(np.int32)))

    for V in (64, 300, 1000, 8194):
        for T, k, p, pen in [(0.8, 30, 0.8, 10.0), (1.0, 10, 0.9, 1.3), (1.3, 0, 0.95, 1.0),
                             (0.5, 1, 0.5, 2.0), (-1.0, V, 1.0, 0.5), (0.8, 200, 0.0, 10.0)]:
            x = g.normal(0, 3, V).astype(np.float32)
            x[g.integers(0, V, 5)] += 12
            hist = g.integers(-3, V + 3, size=min(256, 4 * V))   # incl. out-of-range ids
            add(x, hist, T, k, p, pen)
    # ties, -inf entries, constant rows, min_tokens_to_keep variants
    x = np.round(g.normal(0, 2, 1000)).astype(np.float32)           # many exact ties
    add(x, g.integers(0, 1000, 100), 0.8, 30, 0.8, 10.0)
    x = g.normal(0, 3, 500).astype(np.float32)
    x[g.integers(0, 500, 100)] = -np.inf
    add(x, g.integers(0, 500, 64), 0.8, 0, 0.9, 10.0)
    add(np.zeros(64, np.float32), np.arange(10), 0.8, 5, 0.8, 10.0)
    add(g.normal(0, 3, 300).astype(np.float32), np.arange(0), 0.7, 0, 0.6, 10.0, min_keep=5)
    add(g.normal(0, 3, 300).astype(np.float32), np.arange(0), 0.7, 0, 0.6, 10.0, min_keep=0)

    R = orc.RefOracle()
    out = {}
    n = len(rows)
    Vmax = max(len(r) for r in rows)
    X = np.full((n, Vmax), np.nan, np.float32)
    HIST = []
    OFF = np.zeros(n + 1, np.int64)
    meta = np.zeros((n, 6), np.float64)
    outs = {k: np.full((n, Vmax), np.nan, np.float32) for k in ("temp", "rep", "topk", "topp", "chain")}
    argm = np.zeros(n, np.int32)
    for i, (x, (V, T, k, p, pen, mk, hist)) in enumerate(zip(rows, specs)):
        X[i, :V] = x
        HIST.append(hist)
        OFF[i + 1] = OFF[i] + len(hist)
        meta[i] = (V, T, k, p, pen, mk)
        v = x.copy(); R.temperature(v, T); outs["temp"][i, :V] = v
        v = x.copy(); R.repetition_penalty(v, hist, pen); outs["rep"][i, :V] = v
        v = x.copy(); R.top_k(v, k); outs["topk"][i, :V] = v
        v = x.copy(); R.top_p(v, p, mk); outs["topp"][i, :V] = v
        v = x.copy()
        R.repetition_penalty(v, hist, pen); R.temperature(v, T); R.top_k(v, k); R.top_p(v, p, mk)
        outs["chain"][i, :V] = v
        argm[i] = R.argmax(x)
    np.savez_compressed(os.path.join(HERE, "ref_proc.npz"), x=X, hist=np.concatenate(HIST),
                        hist_off=OFF, meta=meta, argmax=argm, **outs)
    print(f"[ref_proc] {n} rows")


def chain_cases():
    """Multi-step draws through the reference processors + restated draw."""
    R = orc.RefOracle()
    # c0: one stream, 48 steps over a pool of 16 logit rows, history grows.
    g = np.random.default_rng(7)
    pool = wl.normal_logits(g, 16, wl.SEMANTIC_VOCAB, spikes=5)
    hist0 = g.integers(0, 8192, 256).astype(np.int32)
    res = {}
    for mode in ("sample", "greedy"):
        params = wl.make_params(1, greedy=int(mode == "greedy"))
        rng = wl.seed_states(1, 0)
        hist, off = hist0.copy(), np.array([0, 256], np.int64)
        ids = []
        for s in range(48):
            x = np.ascontiguousarray(pool[s % 16:s % 16 + 1])
            t, _ = R.sample_batch(x, wl.SEMANTIC_VOCAB, hist, off, params, rng)
            ids.append(int(t[0]))
            hist, off = wl.append_history(hist, off, t)
        res[f"c0_{mode}_ids"] = np.array(ids, np.int32)
        res[f"c0_{mode}_rng"] = rng.copy()
    res["c0_pool"] = pool
    res["c0_hist0"] = hist0
    # c2: heterogeneous batch, 24 rows, one step, with processed logits.
    b = wl.config2(seed=11, B=24)
    rng = b.rng.copy()
    ids, lg = R.sample_batch(b.logits, b.V, b.hist, b.hist_off, b.params, rng, want_logits=True)
    res.update(c2_logits=b.logits, c2_hist=b.hist, c2_hist_off=b.hist_off,
               c2_params=b.params.view(np.uint8).reshape(-1, 24), c2_rng0=b.rng,
               c2_ids=ids, c2_rng1=rng, c2_out=lg)
    np.savez_compressed(os.path.join(HERE, "ref_chain.npz"), **res)
    print("[ref_chain] c0 48 steps x 2 modes, c2 24 rows")


if __name__ == "__main__":
    orc.build(ref_tree=REF)
    hf_goldens()
    proc_cases()
    chain_cases()
