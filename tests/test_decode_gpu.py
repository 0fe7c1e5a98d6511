"""The device-resident decode step and driver (text2semantic.cpp:167-178 and
:196-373 of the reference), through the C ABI.

A small synthetic model (the forward pass is the identity: the next hidden
states are the next input embeddings) runs DecodeLoop step by step. Every
step is replayed on the CPU from the GPU's own logits: the oracle samples the
unfinished rows with the replayed histories and xorshift64 states, and numpy
does the bookkeeping (stop token, history and latent append, next embedding
as a bf16 add). Ids, states, histories, done flags, next embeddings and
latents must agree bit for bit at every step.
"""
import numpy as np
import pytest

from conftest import load_c4s
from helpers import NTHREADS

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def c4s():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return load_c4s()


def _bf16_add(wl, a, b):
    return wl.bf16_bits(wl.bf16_float(a) + wl.bf16_float(b))


@pytest.mark.parametrize("greedy", [False, True])
def test_decode_loop_matches_cpu_replay(c4s, oracle, greedy):
    wl = c4s.workloads
    B, d, V, steps = 12, 128, 1000, 40
    stop = V - 1
    g = np.random.default_rng(8 + greedy)
    W = wl.bf16_bits(g.normal(0, 0.3, (V, d)).astype(np.float32))
    bias = g.normal(0, 0.5, V).astype(np.float32)
    bias[stop] = 2.5                                  # rows stop at different steps
    gamma = (1 + g.normal(0, 0.1, d)).astype(np.float32)
    beta = g.normal(0, 0.1, d).astype(np.float32)
    emb = wl.bf16_bits(g.normal(0, 1, (V, d)).astype(np.float32))
    pos = wl.bf16_bits(g.normal(0, 0.3, (steps + 1, d)).astype(np.float32))
    params = wl.make_params(B, temperature=0.9, top_k=g.choice([0, 20, 50], B).astype(np.int32),
                            top_p=0.9, repetition_penalty=3.0, greedy=int(greedy))
    dev = torch.device("cuda", 0)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    ctx = c4s.SamplingContext(max_vocab=V, device=0)
    head = dict(weight=t(W.view(np.int16)), bias=t(bias), gamma=t(gamma), beta=t(beta))
    loop = c4s.decode.DecodeLoop(ctx, B, head, t(emb.view(np.int16)), t(pos.view(np.int16)), params, seed=77,
                                 max_new_tokens=steps, stop_token=stop, keep_latents=True)
    # CPU replay state
    rng = wl.seed_states(B, 77)
    hists = [[] for _ in range(B)]
    lats = [[] for _ in range(B)]
    active = np.ones(B, bool)
    hidden = t(wl.bf16_bits(g.normal(0, 1, (B, d)).astype(np.float32)).view(np.int16))
    for s in range(steps):
        h_in = hidden.cpu().numpy().view(np.uint16)
        nxt = loop.step(hidden)
        torch.cuda.synchronize()
        lg = loop.logits.cpu().numpy()
        # sampling replay on the GPU's logits, only the active rows
        off = np.zeros(B + 1, np.int64)
        off[1:] = np.cumsum([len(x) for x in hists])
        flat = np.array([v for x in hists for v in x], np.int32)
        ids, _ = oracle.sample_batch(lg, V, flat, off, params, rng, active=active.astype(np.uint8),
                                     nthreads=NTHREADS)
        assert np.array_equal(loop.ids.cpu().numpy(), ids), s
        assert np.array_equal(loop.rng.cpu().numpy().view(np.uint64), rng), s
        tok_e = np.zeros(B, np.int64)
        for b in range(B):
            if not active[b]:
                continue
            if ids[b] == stop:
                active[b] = False
            else:
                hists[b].append(int(ids[b]))
                lats[b].append(h_in[b].copy())
                tok_e[b] = ids[b]
        assert np.array_equal(loop.active.cpu().numpy().astype(bool), active), s
        want = _bf16_add(wl, emb[tok_e], pos[s + 1][None, :])
        assert np.array_equal(nxt.cpu().numpy().view(np.uint16), want), s
        assert loop.finished() == int((~active).sum()), s
        hidden = nxt                                   # the identity "forward pass"
        if not active.any():
            break
    res = loop.results()
    for b in range(B):
        assert res[b][0].tolist() == hists[b]
        if hists[b]:
            assert np.array_equal(res[b][1], np.stack(lats[b]))
    assert (~active).sum() > 0                        # some rows stopped on the stop token
    err, _ = ctx.status(reset=True)
    assert err == 0


def test_full_history_window_stops_the_row(c4s):
    """A row whose window is full stops and raises C4S_DEVERR_HIST_FULL (a
    host-visible flag; nothing out of bounds is written)."""
    ctx = c4s.SamplingContext(max_vocab=64, device=0)
    dev = torch.device("cuda", 0)
    B, d, cap = 3, 16, 2
    ids = torch.tensor([5, 6, 7], dtype=torch.int32, device=dev)
    active = torch.ones(B, dtype=torch.uint8, device=dev)
    hist = torch.full((B * cap,), -9, dtype=torch.int32, device=dev)
    start = torch.arange(B, dtype=torch.int64, device=dev) * cap
    hlen = torch.tensor([0, 1, 2], dtype=torch.int32, device=dev)
    emb = torch.zeros((64, d), dtype=torch.int16, device=dev)
    pos = torch.zeros(d, dtype=torch.int16, device=dev)
    nxt = torch.empty((B, d), dtype=torch.int16, device=dev)
    done = torch.zeros(1, dtype=torch.int32, device=dev)
    ctx.decode_step(ids, active, 63, hist, start, hlen, cap, emb, pos, nxt, done)
    err, _ = ctx.status(reset=True)
    assert err & 8
    assert hist.cpu().tolist() == [5, -9, -9, 6, -9, -9] or hist.cpu().tolist()[:4] == [5, -9, -9, 6]
    assert hlen.cpu().tolist() == [1, 2, 2]
    assert active.cpu().tolist() == [1, 1, 0]
    assert int(done.item()) == 1
