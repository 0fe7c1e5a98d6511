"""Python host side of the B200 T2S sampling stage.

Two layers, matching the C ABI in include/c4s_sampling.h:

* ``SamplingContext`` -- the batched, device-resident entry points
  (``sample``, ``process``, ``argmax``, ``seed_states``) over torch CUDA
  tensors, stream-ordered on the current torch stream.
* Module-level ``temperature``, ``repetition_penalty``, ``top_k``, ``top_p``,
  ``argmax`` -- the reference's five processors (include/c4tts/t2s.h:82-89,
  src/t2s/sampling.cpp:14-76 of the reference) with the same names, argument
  meaning and in-place behaviour: pass a 1-D float32 CUDA tensor, a float32
  numpy array or a Python list and it is modified in place (argmax returns
  the index).

There is no CPU fallback: if the CUDA library is missing or no sm_100 device
is present every call raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import numpy as np

from . import workloads

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libc4s.so")

STAGE_PENALTY = 1
STAGE_TEMPERATURE = 2
STAGE_TOP_K = 4
STAGE_TOP_P = 8
STAGE_ALL = 15
DEBUG_FORCE_EXACT = 1
DEBUG_FORCE_BINS = 2
DEBUG_FORCE_REFINE = 4
DEBUG_SPLIT_PATH = 8
DEBUG_FAIL_AFTER_ROW = 16
DEBUG_FUSED_PATH = 32
COUNTER_NAMES = ("topp_exact_fallback", "draw_exact_fallback", "topk_radix",
                 "topp_binned", "draw_rowpass", "deferred", "exact_tail")
MAX_VOCAB = 32768
SHARD_CANDIDATES = 64   # candidates per row and vocab shard (C4S_SHARD_CANDIDATES)
MAX_SHARDS = 16
DEVERR_SHARD = 4

_STATUS = {0: "ok", -1: "invalid argument", -2: "CUDA error", -3: "capacity exceeded",
           -4: "device-side error", -5: "device wait timed out", -6: "collective failed"}


class C4SError(RuntimeError):
    """A c4s C-ABI call returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{_STATUS.get(status, status)}: {message}")
        self.status = status


_lib = None
_lib_lock = threading.Lock()


def library() -> C.CDLL:
    """Load lib/libc4s.so (built by __graft_entry__.build()); raise if absent."""
    global _lib
    with _lib_lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(f"c4s CUDA library not built: {LIB_PATH} is missing "
                                   "(run `python -c 'import __graft_entry__ as g; g.build()'`)")
            L = C.CDLL(LIB_PATH)
            vp, i32, i64, u64 = C.c_void_p, C.c_int32, C.c_int64, C.c_uint64
            sig = {
                "c4s_version": ([], C.c_int),
                "c4s_status_string": ([C.c_int], C.c_char_p),
                "c4s_create": ([C.POINTER(vp), i32, i32], C.c_int),
                "c4s_create_sized": ([C.POINTER(vp), i32, i32, i32], C.c_int),
                "c4s_destroy": ([vp], C.c_int),
                "c4s_last_error": ([vp], C.c_char_p),
                "c4s_set_debug": ([vp, i32], C.c_int),
                "c4s_seed_states": ([vp, i32, u64, i64, vp], C.c_int),
                "c4s_sample": ([vp, vp, i32, i32, i64, vp, vp, i64, vp, i32, vp, vp, vp, vp, i64, vp],
                               C.c_int),
                "c4s_process": ([vp, vp, i32, i32, i64, vp, vp, i64, vp, i32, i32, vp], C.c_int),
                "c4s_argmax": ([vp, vp, i32, i32, i64, vp, vp], C.c_int),
                "c4s_get_status": ([vp, vp, vp, i32, vp], C.c_int),
                "c4s_kernel_timing": ([vp, i32], C.c_int),
                "c4s_kernel_times": ([vp, vp, vp, i32], C.c_int),
                "c4s_shard_candidates": ([vp, vp, i32, i32, i64, i32, i32, vp, vp, i64, vp, i32, vp, vp,
                                          vp], C.c_int),
                "c4s_shard_candidates_split": ([vp, vp, i32, i32, i64, i32, vp, vp, i64, vp, i32, vp, vp,
                                                i64, vp], C.c_int),
                "c4s_shard_candidates_sub": ([vp, vp, i32, i32, i64, i32, i32, i32, vp, vp, i64, vp, i32, vp,
                                              vp, i64, vp], C.c_int),
                "c4s_merge_candidates": ([vp, vp, i32, i64, i32, i32, vp, i32, vp, vp, vp, vp], C.c_int),
                "c4s_test_div_rn": ([vp, C.c_float, vp, i64, vp], C.c_int),
                "c4s_sample_windows": ([vp, vp, i32, i32, i64, vp, vp, vp, i64, vp, i32, vp, vp, vp, vp, i64, vp],
                                       C.c_int),
                "c4s_decode_step": ([vp, vp, i32, vp, i32, vp, vp, vp, i32, vp, i32, vp, i32, vp, vp, vp, vp, vp],
                                    C.c_int),
                "c4s_quantize_affine": ([vp, vp, i32, i32, i32, i32, vp, vp, vp, vp], C.c_int),
                "c4s_qgemv": ([vp, vp, i32, i32, vp, vp, vp, i32, i32, i32, vp, vp, vp], C.c_int),
                "c4s_head_logits": ([vp, vp, i32, i32, i64, vp, vp, C.c_float, vp, i32, i64, vp, vp, vp, i64, vp],
                                    C.c_int),
                "c4s_head_sample": ([vp, vp, i32, i32, i64, vp, vp, C.c_float, vp, i32, i64, vp, vp, vp, i64,
                                     vp, vp, i64, vp, i32, vp, vp, vp, vp], C.c_int),
            }
            for name, (args, res) in sig.items():
                f = getattr(L, name)
                f.argtypes = args
                f.restype = res
            _lib = L
        return _lib


def _torch():
    import torch
    return torch


def _dptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def params_tensor(params: np.ndarray, device) -> "torch.Tensor":
    """Upload a ROW_PARAMS_DTYPE array as raw bytes (24 B per row)."""
    torch = _torch()
    assert params.dtype == workloads.ROW_PARAMS_DTYPE
    raw = np.ascontiguousarray(params).view(np.uint8)
    return torch.from_numpy(raw.copy()).to(device)


class SamplingContext:
    """One c4s context (device workspace) bound to a CUDA device.

    ``max_rows`` sizes the workspace for batches of up to that many rows per
    call (None: 4096, about 0.76 GB at max_vocab 8194); larger batches still
    run, in chunks (c4s_create_sized)."""

    def __init__(self, max_vocab: int = workloads.SEMANTIC_VOCAB, device=None, max_rows: int | None = None):
        torch = _torch()
        self.lib = library()
        if device is None:
            device = torch.cuda.current_device()
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        self.max_vocab = max_vocab
        self.max_rows = max_rows
        h = C.c_void_p()
        if max_rows is None:
            rc = self.lib.c4s_create(C.byref(h), max_vocab, self.device.index or 0)
        else:
            rc = self.lib.c4s_create_sized(C.byref(h), max_vocab, int(max_rows), self.device.index or 0)
        if rc != 0:
            raise C4SError(rc, f"c4s_create(max_vocab={max_vocab}, max_rows={max_rows}, device={self.device})")
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            self.lib.c4s_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- helpers --------------------------------------------------------------
    def _check(self, rc: int, what: str):
        if rc != 0:
            msg = self.lib.c4s_last_error(self._h).decode()
            raise C4SError(rc, f"{what}: {msg}")

    def _stream(self, stream):
        torch = _torch()
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        return C.c_void_p(s.cuda_stream)

    def set_debug(self, flags: int):
        self._check(self.lib.c4s_set_debug(self._h, flags), "c4s_set_debug")

    def status(self, reset: bool = False, stream=None):
        """Synchronise and return (device error bits, {counter: value})."""
        err = C.c_uint32(0)
        cnt = (C.c_uint64 * 8)()
        rc = self.lib.c4s_get_status(self._h, C.byref(err), cnt, int(reset), self._stream(stream))
        counters = {n: int(cnt[i]) for i, n in enumerate(COUNTER_NAMES)}
        if rc not in (0, -4, -5):
            self._check(rc, "c4s_get_status")
        return int(err.value), counters

    def kernel_timing(self, enable: bool):
        """Record CUDA events around the fast path's kernels of later calls."""
        self._check(self.lib.c4s_kernel_timing(self._h, int(enable)), "c4s_kernel_timing")

    def kernel_times(self, reset: bool = True):
        """{kernel: (summed device ms, launches)} of the calls recorded so far."""
        ms = (C.c_double * 5)()
        n = (C.c_int64 * 5)()
        self._check(self.lib.c4s_kernel_times(self._h, ms, n, int(reset)), "c4s_kernel_times")
        names = ("order_kernel", "row_kernel", "list_kernel", "defer_kernel", "fused_kernel")
        return {k: (float(ms[i]), int(n[i])) for i, k in enumerate(names)}

    # -- batched entry points -----------------------------------------------------
    def seed_states(self, B: int, seed: int, row_offset: int = 0, out=None, stream=None):
        """int64 CUDA tensor holding the uint64 xorshift states (text2semantic.cpp:292-295)."""
        torch = _torch()
        if out is None:
            out = torch.empty(B, dtype=torch.int64, device=self.device)
        rc = self.lib.c4s_seed_states(_dptr(out), B, seed & (2**64 - 1), row_offset, self._stream(stream))
        self._check(rc, "c4s_seed_states")
        return out

    def sample(self, logits, hist, hist_off, params, rng, active=None, out_ids=None,
               out_logits=None, V: int | None = None, params_stride: int = 1, stream=None):
        """One fused sampling step over the rows of ``logits`` [B, ld].

        hist int32 / hist_off int64 [B+1] (CSR, may be None), params uint8
        [B*24] (or 24 with params_stride=0), rng int64 [B] (advanced in
        place), active uint8 [B] or None. Returns int32 ids [B].
        """
        torch = _torch()
        B, ld = logits.shape
        V = ld if V is None else V
        if out_ids is None:
            out_ids = torch.empty(B, dtype=torch.int32, device=logits.device)
        total = 0 if hist is None else hist.numel()
        rc = self.lib.c4s_sample(
            self._h, _dptr(logits), B, V, logits.stride(0), _dptr(hist), _dptr(hist_off), total,
            _dptr(params), params_stride, _dptr(rng), _dptr(active), _dptr(out_ids),
            _dptr(out_logits), 0 if out_logits is None else out_logits.stride(0), self._stream(stream))
        self._check(rc, "c4s_sample")
        return out_ids

    def sample_windows(self, logits, hist, hist_start, hist_len, params, rng, active=None, out_ids=None,
                       out_logits=None, V: int | None = None, params_stride: int = 1, stream=None):
        """c4s_sample with per-row history windows: hist int32, hist_start int64
        [B], hist_len int32 [B] (row b's ids are hist[start[b]:start[b]+len[b]])."""
        torch = _torch()
        B, ld = logits.shape
        V = ld if V is None else V
        if out_ids is None:
            out_ids = torch.empty(B, dtype=torch.int32, device=logits.device)
        total = 0 if hist is None else hist.numel()
        rc = self.lib.c4s_sample_windows(
            self._h, _dptr(logits), B, V, logits.stride(0), _dptr(hist), _dptr(hist_start), _dptr(hist_len), total,
            _dptr(params), params_stride, _dptr(rng), _dptr(active), _dptr(out_ids), _dptr(out_logits),
            0 if out_logits is None else out_logits.stride(0), self._stream(stream))
        self._check(rc, "c4s_sample_windows")
        return out_ids

    def decode_step(self, ids, active, stop_token: int, hist, hist_start, hist_len, hist_cap: int, emb, pos_row,
                    next_emb, done_count, cur=None, latents=None, stream=None):
        """c4s_decode_step: append ids to the history windows, stop rows on
        stop_token, write next_emb = emb[tok] + pos_row (bf16 bits)."""
        B = ids.shape[0]
        D = emb.shape[1]
        rc = self.lib.c4s_decode_step(
            self._h, _dptr(ids), B, _dptr(active), stop_token, _dptr(hist), _dptr(hist_start), _dptr(hist_len),
            hist_cap, _dptr(emb), emb.shape[0], _dptr(pos_row), D, _dptr(next_emb), _dptr(cur), _dptr(latents),
            _dptr(done_count), self._stream(stream))
        self._check(rc, "c4s_decode_step")

    def quantize_affine(self, w, group: int = 64, bits: int = 8, stream=None):
        """Affine group quantization (MLX's scheme, gpt2.cpp:52-60) of an fp32
        CUDA tensor w [N, K] (out x in): returns (q uint32 as int32 [N, K*bits/32],
        scales fp32 [N, K/group], biases fp32 [N, K/group])."""
        torch = _torch()
        N, K = w.shape
        q = torch.empty((N, K * bits // 32), dtype=torch.int32, device=w.device)
        sc = torch.empty((N, K // group), dtype=torch.float32, device=w.device)
        bi = torch.empty((N, K // group), dtype=torch.float32, device=w.device)
        rc = self.lib.c4s_quantize_affine(self._h, _dptr(w), N, K, group, bits, _dptr(q), _dptr(sc), _dptr(bi),
                                          self._stream(stream))
        self._check(rc, "c4s_quantize_affine")
        return q, sc, bi

    def qgemv(self, x, q, scales, biases, group: int = 64, bits: int = 8, bias_out=None, out=None, stream=None):
        """y = x dequant(q)^T + bias_out (quantized_matmul(transpose=true) + bias,
        gpt2.cpp:61-63); x fp32 [B, K]."""
        torch = _torch()
        B, K = x.shape
        N = q.shape[0]
        if out is None:
            out = torch.empty((B, N), dtype=torch.float32, device=x.device)
        rc = self.lib.c4s_qgemv(self._h, _dptr(x), B, K, _dptr(q), _dptr(scales), _dptr(biases), N, group, bits,
                                _dptr(bias_out), _dptr(out), self._stream(stream))
        self._check(rc, "c4s_qgemv")
        return out

    def head_logits(self, hidden, weight, bias=None, gamma=None, beta=None, eps: float = 1e-5,
                    layer_norm: bool = True, norm_out=None, logits_out=None, stream=None):
        """LM head (text2semantic.cpp:118-121): logits = LayerNorm(hidden) W^T + b
        on the tensor cores. hidden int16/uint16 CUDA tensor of bf16 bits [B, d]
        (or torch.bfloat16), weight bf16 [N, d]; returns fp32 logits [B, N].
        layer_norm=False skips the LayerNorm (a plain linear, nn.cpp:11-16)."""
        torch = _torch()
        B, d = hidden.shape
        N = weight.shape[0]
        dev = hidden.device
        if logits_out is None:
            logits_out = torch.empty((B, N), dtype=torch.float32, device=dev)
        if layer_norm and norm_out is None:
            norm_out = torch.empty((B, d), dtype=torch.int16, device=dev)
        rc = self.lib.c4s_head_logits(self._h, _dptr(hidden), B, d, hidden.stride(0), _dptr(gamma), _dptr(beta),
                                      eps, _dptr(weight), N, weight.stride(0), _dptr(bias),
                                      _dptr(norm_out) if layer_norm else None, _dptr(logits_out),
                                      logits_out.stride(0), self._stream(stream))
        self._check(rc, "c4s_head_logits")
        return logits_out, (norm_out if layer_norm else None)

    def head_sample(self, hidden, weight, bias, gamma, beta, hist, hist_off, params, rng, active=None,
                    out_ids=None, eps: float = 1e-5, norm_out=None, logits_out=None, params_stride: int = 1,
                    stream=None):
        """One decode step's head and sampling (c4s_head_sample); returns
        (ids, logits, normalised states)."""
        torch = _torch()
        B, d = hidden.shape
        N = weight.shape[0]
        dev = hidden.device
        if logits_out is None:
            logits_out = torch.empty((B, N), dtype=torch.float32, device=dev)
        if norm_out is None:
            norm_out = torch.empty((B, d), dtype=torch.int16, device=dev)
        if out_ids is None:
            out_ids = torch.empty(B, dtype=torch.int32, device=dev)
        total = 0 if hist is None else hist.numel()
        rc = self.lib.c4s_head_sample(self._h, _dptr(hidden), B, d, hidden.stride(0), _dptr(gamma), _dptr(beta),
                                      eps, _dptr(weight), N, weight.stride(0), _dptr(bias), _dptr(norm_out),
                                      _dptr(logits_out), logits_out.stride(0), _dptr(hist), _dptr(hist_off), total,
                                      _dptr(params), params_stride, _dptr(rng), _dptr(active), _dptr(out_ids),
                                      self._stream(stream))
        self._check(rc, "c4s_head_sample")
        return out_ids, logits_out, norm_out

    def sample_from_host(self, logits, hist, hist_off, params, rng, out_ids, V: int | None = None,
                         stream=None):
        """One sampling step on HOST (ideally pinned) tensors, like the
        reference's host-vector interface but batched: uploads the step's
        inputs to device staging buffers, samples, and copies the ids and the
        advanced xorshift states back into ``out_ids`` / ``rng``. Asynchronous
        on the current stream; synchronise before reading the host outputs.
        """
        torch = _torch()
        dev = self.device
        key = (logits.shape, hist.numel(), hist_off.numel(), params.numel(), rng.numel())
        st = getattr(self, "_staging", None)
        if st is None or st[0] != key:
            st = (key, dict(
                logits=torch.empty(logits.shape, dtype=torch.float32, device=dev),
                hist=torch.empty(hist.numel(), dtype=torch.int32, device=dev),
                hist_off=torch.empty(hist_off.numel(), dtype=torch.int64, device=dev),
                params=torch.empty(params.numel(), dtype=torch.uint8, device=dev),
                rng=torch.empty(rng.numel(), dtype=torch.int64, device=dev),
                ids=torch.empty(logits.shape[0], dtype=torch.int32, device=dev)))
            self._staging = st
        d = st[1]
        d["logits"].copy_(logits, non_blocking=True)
        d["hist"].copy_(hist, non_blocking=True)
        d["hist_off"].copy_(hist_off, non_blocking=True)
        d["params"].copy_(params, non_blocking=True)
        d["rng"].copy_(rng, non_blocking=True)
        self.sample(d["logits"], d["hist"], d["hist_off"], d["params"], d["rng"], out_ids=d["ids"], V=V,
                    stream=stream)
        out_ids.copy_(d["ids"], non_blocking=True)
        rng.copy_(d["rng"], non_blocking=True)
        return out_ids

    def shard_candidates(self, logits, V: int, vocab_offset: int, hist, hist_off, params,
                         active=None, out=None, V_shard: int | None = None, params_stride: int = 1,
                         stream=None, num_sub: int = 1):
        """Candidates of one vocab shard: ``logits`` [B, ld] holds the shard's
        columns [vocab_offset, vocab_offset + V_shard) of rows of width V.
        Returns int64 [B, 64] raw c4s_candidate records (value, global index);
        with num_sub > 1, [num_sub, B, 64]: the shard's columns as num_sub
        contiguous sub-shards (c4s_shard_candidates_sub)."""
        torch = _torch()
        B, ld = logits.shape
        V_shard = ld if V_shard is None else V_shard
        total = 0 if hist is None else hist.numel()
        if num_sub > 1:
            if out is None:
                out = torch.empty((num_sub, B, SHARD_CANDIDATES), dtype=torch.int64, device=logits.device)
            rc = self.lib.c4s_shard_candidates_sub(
                self._h, _dptr(logits), B, V_shard, logits.stride(0), vocab_offset, V, num_sub, _dptr(hist),
                _dptr(hist_off), total, _dptr(params), params_stride, _dptr(active), _dptr(out),
                out.stride(0), self._stream(stream))
            self._check(rc, "c4s_shard_candidates_sub")
            return out
        if out is None:
            out = torch.empty((B, SHARD_CANDIDATES), dtype=torch.int64, device=logits.device)
        rc = self.lib.c4s_shard_candidates(
            self._h, _dptr(logits), B, V_shard, logits.stride(0), vocab_offset, V, _dptr(hist),
            _dptr(hist_off), total, _dptr(params), params_stride, _dptr(active), _dptr(out),
            self._stream(stream))
        self._check(rc, "c4s_shard_candidates")
        return out

    def shard_candidates_split(self, logits, num_shards: int, hist, hist_off, params, active=None,
                               out=None, V: int | None = None, params_stride: int = 1, stream=None):
        """Candidates of all ``num_shards`` shards of whole rows ``logits``
        [B, ld] in one launch, into ``out`` int64 [G, B, 64] (the gathered layout)."""
        torch = _torch()
        B, ld = logits.shape
        V = ld if V is None else V
        if out is None:
            out = torch.empty((num_shards, B, SHARD_CANDIDATES), dtype=torch.int64, device=logits.device)
        total = 0 if hist is None else hist.numel()
        rc = self.lib.c4s_shard_candidates_split(
            self._h, _dptr(logits), B, V, logits.stride(0), num_shards, _dptr(hist), _dptr(hist_off),
            total, _dptr(params), params_stride, _dptr(active), _dptr(out), out.stride(0),
            self._stream(stream))
        self._check(rc, "c4s_shard_candidates_split")
        return out

    def merge_candidates(self, cand, V: int, params, rng, active=None, out_ids=None,
                         params_stride: int = 1, stream=None):
        """Token ids from gathered candidates ``cand`` int64 [G, B, 64] (shards
        in vocabulary order); advances ``rng`` like ``sample``."""
        torch = _torch()
        G, B, _ = cand.shape
        if out_ids is None:
            out_ids = torch.empty(B, dtype=torch.int32, device=cand.device)
        rc = self.lib.c4s_merge_candidates(
            self._h, _dptr(cand), G, cand.stride(0), B, V, _dptr(params), params_stride, _dptr(rng),
            _dptr(active), _dptr(out_ids), self._stream(stream))
        self._check(rc, "c4s_merge_candidates")
        return out_ids

    def process(self, logits, hist, hist_off, params, stages: int, V: int | None = None,
                params_stride: int = 1, stream=None):
        """Apply the selected processors in place to the rows of ``logits``."""
        B, ld = logits.shape
        V = ld if V is None else V
        total = 0 if hist is None else hist.numel()
        rc = self.lib.c4s_process(self._h, _dptr(logits), B, V, logits.stride(0), _dptr(hist),
                                  _dptr(hist_off), total, _dptr(params), params_stride, stages,
                                  self._stream(stream))
        self._check(rc, "c4s_process")
        return logits

    def argmax(self, logits, V: int | None = None, out=None, stream=None):
        torch = _torch()
        B, ld = logits.shape
        V = ld if V is None else V
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=logits.device)
        rc = self.lib.c4s_argmax(self._h, _dptr(logits), B, V, logits.stride(0), _dptr(out),
                                 self._stream(stream))
        self._check(rc, "c4s_argmax")
        return out


# ---------------------------------------------------------------------------
# The reference's five processors, same names and in-place semantics.
# ---------------------------------------------------------------------------
_default_ctx: dict = {}


def default_context(max_vocab: int = MAX_VOCAB) -> SamplingContext:
    """The calling thread's context on the current device for the one-row
    functions below (sized for one row per call: a few MB, not the 0.76 GB
    of a 4096-row context)."""
    torch = _torch()
    dev = torch.cuda.current_device()
    key = (threading.get_ident(), dev)
    ctx = _default_ctx.get(key)
    if ctx is None:
        ctx = SamplingContext(max_vocab=max_vocab, device=dev, max_rows=1)
        _default_ctx[key] = ctx
    return ctx


def _as_row(logits):
    """(device tensor [1, V], writeback callable) for a CUDA tensor, numpy array or list."""
    torch = _torch()
    if isinstance(logits, torch.Tensor):
        if not logits.is_cuda or logits.dtype != torch.float32 or logits.dim() != 1:
            raise TypeError("expected a 1-D float32 CUDA tensor")
        if not logits.is_contiguous():
            raise ValueError("logits must be contiguous")
        return logits.view(1, -1), (lambda dev: None)
    arr = np.asarray(logits, dtype=np.float32)
    dev = torch.from_numpy(np.ascontiguousarray(arr).reshape(1, -1).copy()).cuda()

    def writeback(d):
        host = d.view(-1).cpu().numpy()
        if isinstance(logits, np.ndarray):
            logits[...] = host
        else:
            logits[:] = host.tolist()
    return dev, writeback


def _run(logits, P: dict, stages: int, prev_tokens=None):
    torch = _torch()
    dev, writeback = _as_row(logits)
    if dev.shape[1] == 0:
        return
    ctx = default_context()
    params = params_tensor(workloads.make_params(1, **P), dev.device)
    hist = hist_off = None
    if prev_tokens is not None:
        h = np.ascontiguousarray(np.asarray(prev_tokens, dtype=np.int64).astype(np.int32))
        hist = torch.from_numpy(h).to(dev.device)
        hist_off = torch.tensor([0, h.size], dtype=torch.int64, device=dev.device)
    ctx.process(dev, hist, hist_off, params, stages, params_stride=0)
    writeback(dev)


_NEUTRAL = dict(temperature=1.0, top_k=0, top_p=1.0, repetition_penalty=1.0, greedy=0,
                min_tokens_to_keep=1)


def temperature(logits, temp: float) -> None:
    """sampling.cpp:14-17: logits /= temp unless temp == 1 or temp <= 0."""
    _run(logits, dict(_NEUTRAL, temperature=temp), STAGE_TEMPERATURE)


def repetition_penalty(logits, prev_tokens, penalty: float) -> None:
    """sampling.cpp:19-28: penalise each distinct in-range id of prev_tokens once."""
    _run(logits, dict(_NEUTRAL, repetition_penalty=penalty), STAGE_PENALTY, prev_tokens)


def top_k(logits, k: int) -> None:
    """sampling.cpp:30-40: mask logits below the k-th largest to -inf."""
    _run(logits, dict(_NEUTRAL, top_k=k), STAGE_TOP_K)


def top_p(logits, p: float, min_tokens_to_keep: int = 1) -> None:
    """sampling.cpp:42-71: nucleus mask with double softmax / cumulative sums."""
    _run(logits, dict(_NEUTRAL, top_p=p, min_tokens_to_keep=min_tokens_to_keep), STAGE_TOP_P)


def argmax(logits) -> int:
    """sampling.cpp:73-76: index of the first maximum."""
    torch = _torch()
    dev, _ = _as_row(logits)
    if dev.shape[1] == 0:
        return 0
    out = default_context().argmax(dev)
    return int(out.cpu()[0])
