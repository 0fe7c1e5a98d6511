"""Test helpers: run the same batch through the CUDA library and the oracle."""
import os

import numpy as np

from conftest import load_c4s

NTHREADS = max(1, min(32, os.cpu_count() or 1))


def to_dev(b, torch, ld_pad=0):
    """Upload a workloads.Batch; returns a dict of CUDA tensors."""
    c4s = load_c4s()
    dev = torch.device("cuda", 0)
    logits = b.logits
    if ld_pad:
        logits = np.zeros((b.B, b.ld + ld_pad), np.float32)
        logits[:, :b.ld] = b.logits
    return dict(
        logits=torch.from_numpy(np.ascontiguousarray(logits)).to(dev),
        hist=torch.from_numpy(np.ascontiguousarray(b.hist, dtype=np.int32)).to(dev),
        hist_off=torch.from_numpy(np.ascontiguousarray(b.hist_off, dtype=np.int64)).to(dev),
        params=c4s.params_tensor(b.params, dev),
        rng=torch.from_numpy(b.rng.view(np.int64).copy()).to(dev),
    )


def gpu_sample(ctx, b, torch, active=None, want_logits=False, ld_pad=0):
    d = to_dev(b, torch, ld_pad)
    out_logits = None
    if want_logits:
        out_logits = torch.empty((b.B, b.V), dtype=torch.float32, device=d["logits"].device)
    act = None if active is None else torch.from_numpy(active.astype(np.uint8)).cuda()
    ids = ctx.sample(d["logits"], d["hist"], d["hist_off"], d["params"], d["rng"], active=act,
                     out_logits=out_logits, V=b.V)
    torch.cuda.synchronize()
    rng = d["rng"].cpu().numpy().view(np.uint64)
    lg = out_logits.cpu().numpy() if want_logits else None
    return ids.cpu().numpy(), rng, lg


def oracle_sample(oracle, b, active=None, want_logits=False):
    rng = b.rng.copy()
    logits = np.ascontiguousarray(b.logits)
    ids, lg = oracle.sample_batch(logits, b.V, b.hist, b.hist_off, b.params, rng, active=active,
                                  want_logits=want_logits, nthreads=NTHREADS)
    return ids, rng, lg


def bits(x):
    return np.ascontiguousarray(x, np.float32).view(np.uint32)
