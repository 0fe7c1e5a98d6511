"""Config 3: the T2S LM head on the tensor cores, then sampling, through the C ABI.

  LayerNorm (nn.cpp:73-83 of the reference): the GPU's bf16 output against a
    float64 restatement on the same inputs, within one bf16 ulp;
  linear + bias (nn.cpp:11-16): the GPU's fp32 logits against a float64 GEMM
    of the SAME bf16 operands (the GPU's normalised states and the bf16
    weights), within the fp32-accumulation bound  2^-14 * sum|y w| + 2^-23 |b|;
  sampling: ids and xorshift64 states from c4s_head_sample equal the oracle's
    on the GPU's logits, bit for bit (the sampling stage's own contract).
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


@pytest.fixture(scope="module")
def ctx(c4s):
    return c4s.SamplingContext(max_vocab=8194, device=0)


def _dev_bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda()


def _ln_ref(wl, hidden, gamma, beta, eps=1e-5):
    x = wl.bf16_float(hidden).astype(np.float64)
    m = x.mean(axis=1, keepdims=True)
    v = ((x - m) ** 2).mean(axis=1, keepdims=True)
    return (x - m) / np.sqrt(v + eps) * gamma.astype(np.float64) + beta.astype(np.float64)


def _check_ln(wl, got_bits, ref):
    got = wl.bf16_float(got_bits).astype(np.float64)
    mag = np.maximum(np.abs(ref), 1e-30)
    ulp = 2.0 ** (np.floor(np.log2(mag)) - 7)              # bf16: 8 significant bits
    assert np.all(np.abs(got - ref) <= ulp * 1.0001), np.max(np.abs(got - ref) / ulp)
    # and almost everywhere the correctly rounded value
    assert np.mean(got_bits == wl.bf16_bits(ref.astype(np.float32))) > 0.99


def _check_gemm(wl, y_bits, weight, bias, got):
    y = wl.bf16_float(y_bits).astype(np.float64)
    w = wl.bf16_float(weight).astype(np.float64)
    ref = y @ w.T + (0.0 if bias is None else bias.astype(np.float64))
    bound = np.abs(y) @ np.abs(w).T * 2.0 ** -14 + (0.0 if bias is None else np.abs(bias) * 2.0 ** -23) + 1e-30
    err = np.abs(got.astype(np.float64) - ref)
    assert np.all(err <= bound), float(np.max(err / bound))


def test_config3_head_and_sampling(c4s, ctx, oracle):
    """B = 256 hidden states of d = 1280 through LayerNorm and the 1280 x 8194
    head, then the config-0 sampling processors and the draw."""
    wl = c4s.workloads
    hb = wl.config3()
    h, W = _dev_bf16(hb.hidden), _dev_bf16(hb.weight)
    g, be, bi = (torch.from_numpy(x).cuda() for x in (hb.gamma, hb.beta, hb.bias))
    hist, off = torch.from_numpy(hb.hist).cuda(), torch.from_numpy(hb.hist_off).cuda()
    params = c4s.params_tensor(hb.params, h.device)
    rng = torch.from_numpy(hb.rng.view(np.int64).copy()).cuda()
    ids, logits, norm = ctx.head_sample(h, W, bi, g, be, hist, off, params, rng)
    torch.cuda.synchronize()
    err, _ = ctx.status(reset=True)
    assert err == 0
    y_bits = norm.cpu().numpy().view(np.uint16)
    _check_ln(wl, y_bits, _ln_ref(wl, hb.hidden, hb.gamma, hb.beta))
    lg = logits.cpu().numpy()
    _check_gemm(wl, y_bits, hb.weight, hb.bias, lg)
    ro = hb.rng.copy()
    io, _ = oracle.sample_batch(np.ascontiguousarray(lg), hb.N, hb.hist, hb.hist_off, hb.params, ro,
                                nthreads=NTHREADS)
    assert np.array_equal(ids.cpu().numpy(), io)
    assert np.array_equal(rng.cpu().numpy().view(np.uint64), ro)


@pytest.mark.parametrize("B,d,N,ldw_pad,ln", [(77, 256, 1000, 0, True), (1, 128, 8194, 0, True),
                                              (130, 192, 520, 64, False), (300, 1280, 8194, 0, True),
                                              (5, 64, 37, 8, False)])
def test_head_shapes(c4s, ctx, B, d, N, ldw_pad, ln):
    """Ragged tiles in both dimensions, strided weights, the head without
    LayerNorm, one row, the smallest K."""
    wl = c4s.workloads
    r = np.random.default_rng(B * 7 + N)
    hidden = wl.bf16_bits(r.normal(0, 1, (B, d)).astype(np.float32))
    weight = np.zeros((N, d + ldw_pad), np.uint16)
    weight[:, :d] = wl.bf16_bits(r.normal(0, 0.05, (N, d)).astype(np.float32))
    bias = r.normal(0, 0.1, N).astype(np.float32)
    gamma = (1 + r.normal(0, 0.1, d)).astype(np.float32)
    beta = r.normal(0, 0.1, d).astype(np.float32)
    h, W = _dev_bf16(hidden), _dev_bf16(weight)[:, :d]
    bi, g, be = (torch.from_numpy(x).cuda() for x in (bias, gamma, beta))
    logits, norm = ctx.head_logits(h, W, bi, g, be, layer_norm=ln)
    torch.cuda.synchronize()
    err, _ = ctx.status(reset=True)
    assert err == 0
    if ln:
        y_bits = norm.cpu().numpy().view(np.uint16)
        _check_ln(wl, y_bits, _ln_ref(wl, hidden, gamma, beta))
    else:
        y_bits = hidden
    _check_gemm(wl, y_bits, weight[:, :d], bias, logits.cpu().numpy())


def test_head_rejects_bad_shapes(c4s, ctx):
    h = torch.zeros((4, 100), dtype=torch.int16, device="cuda")
    W = torch.zeros((8, 100), dtype=torch.int16, device="cuda")
    with pytest.raises(c4s.C4SError):
        ctx.head_logits(h, W, layer_norm=False)              # d not a multiple of 64
    h = torch.zeros((4, 192), dtype=torch.int16, device="cuda")
    W = torch.zeros((8, 192), dtype=torch.int16, device="cuda")
    with pytest.raises(c4s.C4SError):
        ctx.head_logits(h, W, layer_norm=True)               # LayerNorm needs d % 128 == 0
