"""Quantized decode GEMVs (gpt2.cpp:52-73 of the reference; int8 group 64 is
the product default, apps/c4tts_cli.cpp:300-306), through the C ABI.

  quantizer: codes, scales and biases equal a numpy restatement of the affine
    scheme (float32 arithmetic, round half to even) bit for bit, and the
    dequantized weights are within half a step of the originals;
  GEMV: y = x dequant(q)^T + b against float64 on the same quantized
    weights, within the fp32-accumulation bound 2^-13 sum |x||w| (+ 2^-23 |b|).
"""
import numpy as np
import pytest

from conftest import load_c4s

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def c4s():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return load_c4s()


@pytest.fixture(scope="module")
def ctx(c4s):
    return c4s.SamplingContext(max_vocab=64, device=0)


def quantize_ref(w, group, bits):
    N, K = w.shape
    g = w.reshape(N, K // group, group)
    mn = g.min(axis=2)
    mx = g.max(axis=2)
    qmax = np.float32((1 << bits) - 1)
    scale = ((mx - mn) / qmax).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.rint((g - mn[:, :, None]) / scale[:, :, None]).astype(np.float32)
    q = np.where(scale[:, :, None] > 0, np.clip(q, 0, qmax), 0).astype(np.uint32)
    per = 32 // bits
    qw = q.reshape(N, K // per, per)
    words = np.zeros((N, K // per), np.uint32)
    for e in range(per):
        words |= qw[:, :, e] << np.uint32(bits * e)
    return words, scale, mn.astype(np.float32), q.reshape(N, K)


@pytest.mark.parametrize("N,K,group,bits", [(3840, 1280, 64, 8), (1280, 5120, 64, 8), (515, 1280, 64, 4),
                                            (300, 256, 32, 8), (129, 512, 128, 4)])
def test_quantizer_matches_restatement(c4s, ctx, N, K, group, bits):
    r = np.random.default_rng(N + K)
    w = (r.normal(0, 0.02, (N, K)) * np.where(r.random((N, K)) < 0.01, 10, 1)).astype(np.float32)
    w[0, :group] = 0.25                                # a constant group: scale 0, q 0
    q, sc, bi = ctx.quantize_affine(torch.from_numpy(w).cuda(), group, bits)
    qr, scr, bir, codes = quantize_ref(w, group, bits)
    assert np.array_equal(q.cpu().numpy().view(np.uint32), qr)
    assert np.array_equal(sc.cpu().numpy(), scr)
    assert np.array_equal(bi.cpu().numpy(), bir)
    deq = (codes.reshape(N, K // group, group) * scr[:, :, None].astype(np.float64) + bir[:, :, None]).reshape(N, K)
    step = np.repeat(scr, group, axis=1).astype(np.float64)
    # half a step, plus the float32 rounding of (w - bias) / scale before rint
    assert np.all(np.abs(deq - w) <= step * (0.5 + 2.0 ** -12) + 1e-12)


@pytest.mark.parametrize("B", [1, 3, 4, 6])
@pytest.mark.parametrize("N,K,group,bits", [(3840, 1280, 64, 8), (1280, 5120, 64, 8), (5120, 1280, 64, 4),
                                            (77, 256, 32, 4), (200, 512, 128, 8)])
def test_qgemv_against_float64(c4s, ctx, B, N, K, group, bits):
    r = np.random.default_rng(B * 1000 + N)
    w = r.normal(0, 0.02, (N, K)).astype(np.float32)
    x = r.normal(0, 1, (B, K)).astype(np.float32)
    bias = r.normal(0, 0.1, N).astype(np.float32)
    q, sc, bi = ctx.quantize_affine(torch.from_numpy(w).cuda(), group, bits)
    y = ctx.qgemv(torch.from_numpy(x).cuda(), q, sc, bi, group, bits, bias_out=torch.from_numpy(bias).cuda())
    torch.cuda.synchronize()
    _, scr, bir, codes = quantize_ref(w, group, bits)
    deq = (codes.reshape(N, K // group, group) * scr[:, :, None].astype(np.float64) + bir[:, :, None]).reshape(N, K)
    ref = x.astype(np.float64) @ deq.T + bias
    bound = np.abs(x.astype(np.float64)) @ np.abs(deq).T * 2.0 ** -13 + np.abs(bias) * 2.0 ** -23 + 1e-30
    err = np.abs(y.cpu().numpy().astype(np.float64) - ref)
    assert np.all(err <= bound), float(np.max(err / bound))


def test_qgemv_rejects_bad_shapes(c4s, ctx):
    x = torch.zeros((1, 100), device="cuda")
    q = torch.zeros((4, 25), dtype=torch.int32, device="cuda")
    s = torch.zeros((4, 2), device="cuda")
    with pytest.raises(c4s.C4SError):
        ctx.qgemv(x, q, s, s, 64, 8)                     # K not a multiple of the group
    with pytest.raises(c4s.C4SError):
        ctx.quantize_affine(torch.zeros((4, 128), device="cuda"), 64, 3)
