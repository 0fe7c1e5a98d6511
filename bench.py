#!/usr/bin/env python3
"""Benchmark of the T2S sampling stage on B200 (one process per GPU).

Workload (the configuration the headline metric is quoted
on): per GPU a batch of B=4096 rows of V=8194 fp32 logits ~N(0, 3^2), ragged
token histories with lengths U[0, 2048], per-row temperature U[0.5, 1.2],
top_k from {0, 20, 50, 200}, top_p U[0.6, 1.0], repetition penalty
U[1, 10], sample mode. A step is one fused sampling pass over the batch
(one c4s_sample call). Inputs are seeded synthetic data; a pool of 3 batches
(3 x 151 MB, larger than the 126 MB L2) is rotated so that no step reads
cache-resident logits.

Rows are independent, so N GPUs shard rows with no collective on the data
path (weak scaling: each rank samples its own 4096-row block of a
4096*N-row batch, seeded with its global row offset).

  value   sampled tokens/s over all ranks, inputs resident in HBM
  e2e     the same through SamplingContext.sample_from_host with pinned host
          buffers: H2D of the step's logits/history/params/states, sampling,
          D2H of ids and states inside the timed region
  b1_p50_us   p50 latency of one B=1 decode step (config 0), CUDA-graph replay

`--impl reference` times the reference's CPU implementation of the same step
(its own sampling.cpp compiled from source plus the restated draw, or the C
oracle port where that build is absent) on all host threads.
"""
import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--rows", type=int, default=4096, help="rows per GPU")
    ap.add_argument("--pool", type=int, default=3)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--b1-steps", type=int, default=500)
    ap.add_argument("--workload", choices=["c2", "c3", "c4", "qgemv"], default="c2",
                    help="c2: the headline row-sharded batch; c3: LM head (LayerNorm + tcgen05 GEMM) + "
                         "sampling, B=256 x d=1280 x V=8194; c4: vocab-sharded B=512 x V=65536 "
                         "(8 shards on one GPU, or one shard per rank with an NCCL all-gather)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--profile-steps", type=int, default=0,
                    help="only run this many steps of the main loop (for ncu), print nothing")
    ap.add_argument("--profile-config", choices=["c2", "c0", "c2k0", "c2k20"], default="c2",
                    help="with --profile-steps: c2 = config-2 rows (--rows), c0 = one config-0 row, "
                         "c2k0 / c2k20 = config-2 rows all without top-k / all with top_k 20")
    return ap.parse_args()


def load_pkg():
    import __graft_entry__ as ge
    return ge._load_pkg()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, phys_index):
        self.idx = phys_index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.flush()
        rows = []
        with open(self.f.name) as fh:
            for line in fh:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9 or parts[0] != str(self.idx):
                    continue
                rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[j] for r in rows for j in range(4) if r[5 + j].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


def profiled_traffic(B, profile="row_kernel_config2_dram.txt"):
    """DRAM bytes (read + write) of one launch of the profiled kernel at B rows,
    from the committed ncu summary of the same workload (scaled by rows if B
    differs)."""
    path = os.path.join(ROOT, "profiles", profile)
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    _, v, rows = line.split()
                    return float(v) * B / float(rows)
    except OSError:
        pass
    return None


def phys_index(local):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = vis.split(",")
        if local < len(ids) and ids[local].strip().isdigit():
            return int(ids[local])
    return local


# ---------------------------------------------------------------------------
WORKLOAD_C2 = ("config2: B=4096 V=8194 fp32 logits ~N(0,9), ragged history U[0,2048], per-row T U[0.5,1.2], "
               "top_k {0,20,50,200}, top_p U[0.6,1.0], penalty U[1,10]")


def c2_config(rows, world):
    """The workload dict both arms print (identical for the same launch)."""
    return {"workload": WORKLOAD_C2, "global_batch": rows * world, "rows_per_gpu": rows, "V": 8194,
            "l2": "inputs > L2 (a pool of 3 batches rotated on the GPU)"}


def cpu_serial_rows_per_s(c4s, batch, rows=192):
    """The reference's CPU path on ONE thread, rows processed one after the
    other as generate_batch loops them (text2semantic.cpp:303), on the first
    `rows` rows of the batch (a bounded sample)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    impl, kind = (orc.RefOracle(), "reference") if orc.RefOracle.available() else (orc.Oracle(), "port")
    n = min(rows, batch.B)
    sub = c4s.workloads.Batch(np.ascontiguousarray(batch.logits[:n]), batch.V, batch.hist, batch.hist_off[:n + 1],
                              batch.params[:n], batch.rng[:n].copy())
    t0 = time.perf_counter()
    impl.sample_batch(sub.logits, sub.V, sub.hist, sub.hist_off, sub.params, sub.rng, nthreads=1)
    el = time.perf_counter() - t0
    return n / el, kind, n


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def cpu_reference_rows_per_s(c4s, seconds, rows_cap=4096, batch=None):
    """Time the reference CPU path (compiled reference, else the C port) on
    config-2 rows with all host threads; returns (rows/s, kind, threads, rows)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    if orc.RefOracle.available():
        impl, kind = orc.RefOracle(), "reference"
    else:
        impl, kind = orc.Oracle(), "port"
    threads = os.cpu_count() or 1
    b = batch or c4s.workloads.config2(seed=2, B=rows_cap)
    done, t0 = 0, time.perf_counter()
    chunk = min(b.B, max(threads * 8, 256))
    while True:
        s = done % b.B
        e = min(b.B, s + chunk)
        sub = c4s.workloads.Batch(np.ascontiguousarray(b.logits[s:e]), b.V, b.hist,
                                  b.hist_off[s:e + 1], b.params[s:e], b.rng[s:e].copy())
        impl.sample_batch(sub.logits, sub.V, sub.hist, sub.hist_off, sub.params, sub.rng, nthreads=threads)
        done += e - s
        el = time.perf_counter() - t0
        if el >= seconds and done >= chunk:
            return done / el, kind, threads, done


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    c4s = load_pkg()
    b = c4s.workloads.config2(seed=2, B=args.rows)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    impl, kind = (orc.RefOracle(), "reference") if orc.RefOracle.available() else (orc.Oracle(), "port")
    threads = os.cpu_count() or 1

    def step():
        rng = b.rng.copy()
        impl.sample_batch(b.logits, b.V, b.hist, b.hist_off, b.params, rng, nthreads=threads)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    v = args.rows * args.steps / el
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    sv, _, sn = cpu_serial_rows_per_s(c4s, b)
    line = {
        "impl": "reference", "metric": "sampled tokens/s (B=4096, V=8194, config 2)", "value": v,
        "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el * 1e3 / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32+f64", "data": "synthetic",
        "config": c2_config(args.rows, world),
        "execution": f"host CPU, OpenMP over rows, {threads} threads, rank 0 only",
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": kind,
                         "sample": f"full {args.rows}-row config-2 batch per step, OpenMP over rows "
                                   f"with {threads} threads",
                         "serial_1core": {"value": sv, "unit": "tokens/s",
                                          "sample": f"first {sn} rows of the batch, one thread, rows one after "
                                                    "the other (text2semantic.cpp:303)"},
                         "cpu_model": cpu_model()},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def gather_ranks(x):
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        if world == 1:
            return [x]
        out = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(out, t)
        return [float(o.item()) for o in out]

    c4s = load_pkg()
    wl = c4s.workloads
    B = args.rows
    ctx = c4s.SamplingContext(max_vocab=wl.SEMANTIC_VOCAB, device=local)
    stream = torch.cuda.current_stream(dev)

    # ---- inputs: pool of batches, this rank's block of the global batch ----
    pool, host = [], []
    if args.profile_steps and args.profile_config == "c0":
        B = 1
    for k in range(args.pool):
        if args.profile_steps and args.profile_config == "c0":
            b = wl.config0(seed=k)
        else:
            b = wl.config2(seed=2 + k, B=B, row_offset=rank * B)
            if args.profile_steps and args.profile_config in ("c2k0", "c2k20"):
                b.params["top_k"][:] = 0 if args.profile_config == "c2k0" else 20
        pool.append(dict(
            logits=torch.from_numpy(b.logits).to(dev),
            hist=torch.from_numpy(b.hist).to(dev),
            hist_off=torch.from_numpy(b.hist_off).to(dev),
            params=c4s.params_tensor(b.params, dev),
            rng=torch.from_numpy(b.rng.view(np.int64).copy()).to(dev),
            bytes=wl.algorithmic_bytes(b.V, b.hist_off, B)))
        host.append(b)
    ids = torch.empty(B, dtype=torch.int32, device=dev)

    def step(s):
        p = pool[s % len(pool)]
        ctx.sample(p["logits"], p["hist"], p["hist_off"], p["params"], p["rng"], out_ids=ids)

    if args.profile_steps:
        for s in range(args.profile_steps):
            step(s)
        torch.cuda.synchronize()
        return

    for s in range(max(3, args.warmup)):
        step(s)
    torch.cuda.synchronize()

    # ---- clocks under sustained load (~2 s of back-to-back steps) ----
    clk = ClockSampler(phys_index(local))
    t_end = time.time() + 2.0
    s = 0
    while time.time() < t_end:
        for _ in range(50):
            step(s)
            s += 1
        torch.cuda.synchronize()

    # ---- timed region: exactly K steps ----
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s in range(args.steps):
        step(s)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = clk.stop()
    my_ms = e0.elapsed_time(e1)
    ms = max_over_ranks(my_ms)
    per_rank_ms = gather_ranks(my_ms)
    ms_per_step = ms / args.steps
    rows_total = B * world * args.steps
    value = rows_total / (ms / 1e3)
    err, counters = ctx.status(reset=True)

    # ---- strong scaling (N > 1): the one 4096-row config-2 batch split into
    # contiguous blocks of 4096/N rows, one per rank ----
    strong = None
    if world > 1 and B % world == 0:
        Bs = B // world
        sp = []
        for k in range(args.pool):
            bs = wl.config2(seed=2 + k, B=B)              # the same global batch on every rank
            r0 = rank * Bs
            sub = wl.Batch(np.ascontiguousarray(bs.logits[r0:r0 + Bs]), bs.V, bs.hist,
                           bs.hist_off[r0:r0 + Bs + 1], bs.params[r0:r0 + Bs], bs.rng[r0:r0 + Bs].copy())
            sp.append(dict(logits=torch.from_numpy(sub.logits).to(dev), hist=torch.from_numpy(sub.hist).to(dev),
                           hist_off=torch.from_numpy(sub.hist_off).to(dev),
                           params=c4s.params_tensor(sub.params, dev),
                           rng=torch.from_numpy(sub.rng.view(np.int64).copy()).to(dev)))
        ids_s = torch.empty(Bs, dtype=torch.int32, device=dev)

        def sstep(s):
            p = sp[s % len(sp)]
            ctx.sample(p["logits"], p["hist"], p["hist_off"], p["params"], p["rng"], out_ids=ids_s)

        for s in range(max(3, args.warmup)):
            sstep(s)
        torch.cuda.synchronize()
        barrier()
        e0.record(stream)
        for s in range(args.steps):
            sstep(s)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        my_sms = e0.elapsed_time(e1)
        sms = max_over_ranks(my_sms)
        strong = {"global_batch": B, "rows_per_gpu": Bs, "value": B * args.steps / (sms / 1e3),
                  "unit": "tokens/s", "ms_per_step": sms / args.steps,
                  "per_rank_ms_per_step": [t / args.steps for t in gather_ranks(my_sms)],
                  "scaling": "strong"}

    # ---- per-kernel device time: the same K steps again with CUDA events between
    # the launches (order pre-pass -> row kernel -> list kernel -> general path,
    # per 4096-row chunk) ----
    ctx.kernel_timing(True)
    ctx.kernel_times(reset=True)
    for s in range(args.steps):
        step(s)
    kt = ctx.kernel_times(reset=True)
    ctx.kernel_timing(False)
    launches_per_step = sum(n for _, n in kt.values()) // args.steps
    kernels = {k: {"ms_per_launch": ms / max(n, 1), "launches": n,
                   "share": ms / max(sum(m for m, _ in kt.values()), 1e-12)} for k, (ms, n) in kt.items()}

    # ---- roofline of the dominant kernel: the row kernel moves every logit,
    # history id and per-row record (the list and general kernels only touch
    # candidate lists) ----
    alg_bytes = float(np.mean([p["bytes"] for p in pool]))
    hbm_peak, peak_kind = peaks()
    dom = "fused_kernel" if kernels["fused_kernel"]["launches"] else "row_kernel"
    row_ms = kernels[dom]["ms_per_launch"]
    achieved_gbs = alg_bytes / (row_ms / 1e3) / 1e9
    step_gbs = alg_bytes / (ms_per_step / 1e3) / 1e9
    traffic = profiled_traffic(B)

    # ---- e2e through the public host-buffer API ----
    e2e = None
    if not args.no_e2e:
        hp = []
        for b in host:
            hp.append(dict(
                logits=torch.from_numpy(b.logits).pin_memory(),
                hist=torch.from_numpy(b.hist).pin_memory(),
                hist_off=torch.from_numpy(b.hist_off).pin_memory(),
                params=torch.from_numpy(np.ascontiguousarray(b.params).view(np.uint8).copy()).pin_memory(),
                rng=torch.from_numpy(b.rng.view(np.int64).copy()).pin_memory()))
        ids_h = torch.empty(B, dtype=torch.int32).pin_memory()

        def hstep(s):
            p = hp[s % len(hp)]
            ctx.sample_from_host(p["logits"], p["hist"], p["hist_off"], p["params"], p["rng"], ids_h)

        for s in range(3):
            hstep(s)
        torch.cuda.synchronize()
        barrier()
        e0.record(stream)
        for s in range(args.steps):
            hstep(s)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        ms_e2e = max_over_ranks(e0.elapsed_time(e1))
        h2d = int(np.mean([sum(t.numel() * t.element_size() for t in p.values()) for p in hp]))
        d2h = B * 4 + B * 8
        e2e = {"value": B * world * args.steps / (ms_e2e / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "ms_per_step": ms_e2e / args.steps}

    # ---- B=1 decode-step latency (config 0), CUDA graph replay and eager ----
    b1 = None
    if rank == 0:
        b0 = wl.config0()
        d0 = dict(logits=torch.from_numpy(b0.logits).to(dev), hist=torch.from_numpy(b0.hist).to(dev),
                  hist_off=torch.from_numpy(b0.hist_off).to(dev), params=c4s.params_tensor(b0.params, dev),
                  rng=torch.from_numpy(b0.rng.view(np.int64).copy()).to(dev))
        id0 = torch.empty(1, dtype=torch.int32, device=dev)

        def s1():
            ctx.sample(d0["logits"], d0["hist"], d0["hist_off"], d0["params"], d0["rng"], out_ids=id0)

        def lat(fn, n):
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
            for a, bb in ev:
                a.record()
                fn()
                bb.record()
            torch.cuda.synchronize()
            return [a.elapsed_time(bb) * 1e3 for a, bb in ev]

        for _ in range(20):
            s1()
        eager = lat(s1, args.b1_steps)
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            s1()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize()
        with torch.cuda.graph(g):
            s1()
        for _ in range(20):
            g.replay()
        graph = lat(g.replay, args.b1_steps)
        # a device-resident decode loop: a graph of GS dependent steps (each
        # step reads the xorshift state the previous one wrote), replayed;
        # per-step GPU time = replay time / GS, launch overhead amortised
        GS = 64
        g64 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g64):
            for _ in range(GS):
                s1()
        for _ in range(5):
            g64.replay()
        steps64 = [t / GS for t in lat(g64.replay, max(20, args.b1_steps // 10))]
        b1 = {"graph_step_p50_us": statistics.median(steps64), "graph_steps_per_replay": GS,
              "single_replay_p50_us": statistics.median(graph), "eager_p50_us": statistics.median(eager),
              "steps": args.b1_steps,
              "note": "graph_step: GPU time per step inside a captured 64-step loop; single_replay and "
                      "eager: event-to-event time around one host launch (host launch overhead included)"}
        del g, g64

    # ---- config 1 (B=64 streams): GPU time per step in a captured 64-step loop ----
    c1 = None
    if rank == 0:
        bc1 = wl.config1()
        dc1 = dict(logits=torch.from_numpy(bc1.logits).to(dev), hist=torch.from_numpy(bc1.hist).to(dev),
                   hist_off=torch.from_numpy(bc1.hist_off).to(dev), params=c4s.params_tensor(bc1.params, dev),
                   rng=torch.from_numpy(bc1.rng.view(np.int64).copy()).to(dev))
        idc1 = torch.empty(bc1.B, dtype=torch.int32, device=dev)

        def s64(s):
            ctx.sample(dc1["logits"], dc1["hist"], dc1["hist_off"], dc1["params"], dc1["rng"], out_ids=idc1)

        c1 = {"us_per_step": graph_ms_per_step(torch, s64, 64, 5, stream) * 1e3, "rows": bc1.B,
              "timing": "CUDA-graph replay of 64 dependent steps"}

    # ---- CPU baseline (rank 0, N=1 only) ----
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, kind, threads, nrows = cpu_reference_rows_per_s(c4s, args.cpu_seconds, batch=host[0])
        sv, _, sn = cpu_serial_rows_per_s(c4s, host[0])
        cpu = {"value": v, "unit": "tokens/s", "cores": threads, "kind": kind,
               "sample": f"{nrows} rows of the config-2 batch (first {min(B, nrows)} rows, wrapping), "
                         f"OpenMP over rows, {threads} host threads, ~{args.cpu_seconds:.0f} s",
               "serial_1core": {"value": sv, "unit": "tokens/s",
                                "sample": f"first {sn} rows of the batch, one thread, rows one after the other "
                                          "(text2semantic.cpp:303)"},
               "cpu_model": cpu_model()}

    if rank == 0:
        line = {
            "metric": "sampled tokens/s (B=4096, V=8194, config 2)",
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32+f64", "data": "synthetic",
            "config": c2_config(B, world),
            "execution": f"rows x{world} (no collective), pool of {args.pool} batches rotated",
            "per_rank_ms_per_step": [t / args.steps for t in per_rank_ms],
            "strong": strong,
            "c1": c1,
            "b1_p50_us": None if b1 is None else b1["graph_step_p50_us"],
            "b1": b1,
            "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved_gbs / hbm_peak, "traffic": traffic,
                         "kernel": dom, "peak_kind": peak_kind, "alg_bytes_per_launch": alg_bytes,
                         "whole_step_achieved": step_gbs, "whole_step_frac": step_gbs / hbm_peak},
            "kernels": kernels,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
            "device_errors": err,
            "path_counters": counters,
        }
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


def run_vocab_sharded(args):
    """Config 4: every row's 65536-wide vocabulary split into contiguous
    shards. N=1: 8 shards on one GPU (candidate blocks written straight into
    the gathered layout); N>1: shard r on rank r, candidates all-gathered over
    NCCL, every rank merging the same ids. Strong scaling (the batch is fixed)."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    c4s = load_pkg()
    wl = c4s.workloads
    ctx = c4s.SamplingContext(max_vocab=wl.SEMANTIC_VOCAB, device=local)
    stream = torch.cuda.current_stream(dev)
    B, V = 512, wl.VOCAB_SHARDED_V
    voff, width = c4s.vocab_shard.shard_vocab(V, rank, world) if world > 1 else (0, V)
    # candidate blocks: 8 of 8192 columns at every N (N > 1: each rank's shard as sub-shards)
    nsub = c4s.vocab_shard.sub_shards(c4s.vocab_shard.shard_vocab(V, 0, world)[1], world) if world > 1 else 1
    G = 8 if world == 1 else world * nsub
    shard_bytes = B * width * 4
    npool = max(3, -(-300_000_000 // shard_bytes))   # > 2x the 126 MB L2 across the pool
    pool = []
    for k in range(npool):
        b = wl.config4(seed=4 + k, B=B, V=V)
        pool.append(dict(
            logits=torch.from_numpy(np.ascontiguousarray(b.logits[:, voff:voff + width])).to(dev),
            hist=torch.from_numpy(b.hist).to(dev), hist_off=torch.from_numpy(b.hist_off).to(dev),
            params=c4s.params_tensor(b.params, dev),
            rng=torch.from_numpy(b.rng.view(np.int64).copy()).to(dev),
            H=int(b.hist_off[-1])))
    ids = torch.empty(B, dtype=torch.int32, device=dev)
    cand = torch.empty((G, B, c4s.sampling.SHARD_CANDIDATES), dtype=torch.int64, device=dev)

    def step(s):
        p = pool[s % npool]
        if world == 1:
            c4s.vocab_shard.sample_vocab_split(ctx, p["logits"], G, p["hist"], p["hist_off"], p["params"],
                                               p["rng"], out_ids=ids, cand_out=cand, V=V)
        else:
            c4s.vocab_shard.sample_vocab_sharded(ctx, p["logits"], V, p["hist"], p["hist_off"],
                                                 p["params"], p["rng"], out_ids=ids, cand_out=cand)

    def max_over_ranks(x):
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for s in range(max(3, args.warmup)):
        step(s)
    torch.cuda.synchronize()
    # clocks under sustained load: ~2 s of back-to-back steps, then the timed region
    clk = ClockSampler(phys_index(local))
    t_end = time.time() + 2.0
    s = 0
    while time.time() < t_end:
        for _ in range(50):
            step(s)
            s += 1
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s in range(args.steps):
        step(s)
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = clk.stop()
    ms = max_over_ranks(e0.elapsed_time(e1))
    err, _ = ctx.status(reset=True)
    # the shard kernel alone (the only kernel that reads the logits), same inputs,
    # launched back to back between one pair of events on the launching stream
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    nshard = G if world == 1 else nsub   # shards the one shard-kernel launch works

    def shard_launch(s):
        p = pool[s % npool]
        if world == 1:
            ctx.shard_candidates_split(p["logits"], G, p["hist"], p["hist_off"], p["params"], out=cand, V=V)
        elif nsub == 1:
            ctx.shard_candidates(p["logits"], V, voff, p["hist"], p["hist_off"], p["params"], out=cand[rank],
                                 V_shard=width)
        else:
            ctx.shard_candidates(p["logits"], V, voff, p["hist"], p["hist_off"], p["params"],
                                 out=cand[rank * nsub:(rank + 1) * nsub], V_shard=width, num_sub=nsub)

    for s in range(3):
        shard_launch(s)
    torch.cuda.synchronize()
    ev[0].record(stream)
    for s in range(args.steps):
        shard_launch(s)
    ev[1].record(stream)
    torch.cuda.synchronize()
    shard_ms = ev[0].elapsed_time(ev[1]) / args.steps
    H = sum(p["H"] for p in pool) / npool
    alg = B * width * 4 + nshard * (4 * H + B * (8 + 24)) + nshard * B * 64 * 8
    achieved = alg / (shard_ms / 1e3) / 1e9
    hbm_peak, peak_kind = peaks()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # the reference's CPU path on whole 65536-wide rows of the same workload
        v, kind, threads, nrows = cpu_reference_rows_per_s(c4s, args.cpu_seconds,
                                                           batch=wl.config4(seed=4, B=B, V=V))
        cpu = {"value": v, "unit": "tokens/s", "cores": threads, "kind": kind,
               "sample": f"{nrows} whole rows of the config-4 batch (V=65536, wrapping), "
                         f"OpenMP over rows, {threads} host threads, ~{args.cpu_seconds:.0f} s"}
    if rank == 0:
        line = {
            "metric": "sampled tokens/s (B=512, V=65536, vocab-sharded, config 4)",
            "value": B * args.steps / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32+f64", "data": "synthetic",
            "config": {"workload": "config4: B=512 V=65536 fp32 logits ~N(0,9), history 1024/row, "
                                   "T 0.8, penalty 10, global top_k 50 / top_p 0.9",
                       "shards": G, "shard_width": V // G,
                       "parallelism": "8 shards on 1 GPU" if world == 1 else
                                      f"vocab x{world} ({nsub} sub-shards per rank), NCCL all-gather of 64 "
                                      f"candidates/row/sub-shard",
                       "l2": f"pool of {npool} batches rotated (inputs > 2x L2)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak,
                         "traffic": profiled_traffic(B, "vocab_sharded_config4.txt") if world == 1 else None,
                         "kernel": "shard_kernel",
                         "peak_kind": peak_kind, "alg_bytes_per_launch": alg},
            "shard_kernel_ms_per_step": shard_ms,
            "cpu_baseline": cpu,
            "gpu_launches": 2 * args.steps,
            "clocks": clocks, "device_errors": err,
        }
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


def graph_ms_per_step(torch, step, nsteps, reps, stream):
    """GPU time per step of `step(s)` for s in range(nsteps), captured once in
    a CUDA graph and replayed `reps` times between CUDA events: small steps
    are timed without the host's per-launch overhead."""
    side = torch.cuda.Stream()
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        for s in range(nsteps):
            step(s)
    stream.wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for s in range(nsteps):
            step(s)
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (reps * nsteps)
    del g
    return ms


def tensor_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), "measured (burst)"
    return 1590.0, "fallback"


def run_head(args):
    """Config 3: per step LayerNorm + the 1280 x 8194 head GEMM on tcgen05 +
    the sampling step, B=256 rows (c4s_head_sample). Weights and hidden states
    rotate through a pool larger than L2 (a decode step reads the head weights
    from HBM once)."""
    import torch

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    c4s = load_pkg()
    wl = c4s.workloads
    ctx = c4s.SamplingContext(max_vocab=wl.SEMANTIC_VOCAB, device=local)
    stream = torch.cuda.current_stream(dev)
    hb = wl.config3()
    B, d, N = hb.B, hb.hidden.shape[1], hb.N
    wbytes = N * d * 2
    npool = max(3, -(-300_000_000 // wbytes))        # > 2x the 126 MB L2
    g = np.random.default_rng(77)
    pool = []
    for k in range(npool):
        Wk = hb.weight if k == 0 else wl.bf16_bits(g.normal(0, 0.02, size=(N, d)).astype(np.float32))
        hk = hb.hidden if k == 0 else wl.bf16_bits(g.normal(0, 1, size=(B, d)).astype(np.float32))
        pool.append(dict(W=torch.from_numpy(Wk.view(np.int16)).to(dev), h=torch.from_numpy(hk.view(np.int16)).to(dev)))
    gamma, beta, bias = (torch.from_numpy(x).to(dev) for x in (hb.gamma, hb.beta, hb.bias))
    hist, off = torch.from_numpy(hb.hist).to(dev), torch.from_numpy(hb.hist_off).to(dev)
    params = c4s.params_tensor(hb.params, dev)
    rng = torch.from_numpy(hb.rng.view(np.int64).copy()).to(dev)
    ids = torch.empty(B, dtype=torch.int32, device=dev)
    logits = torch.empty((B, N), dtype=torch.float32, device=dev)
    norm = torch.empty((B, d), dtype=torch.int16, device=dev)

    def step(s):
        p = pool[s % npool]
        ctx.head_sample(p["h"], p["W"], bias, gamma, beta, hist, off, params, rng, out_ids=ids,
                        norm_out=norm, logits_out=logits)

    def gemm(s):
        p = pool[s % npool]
        ctx.head_logits(norm, p["W"], bias, layer_norm=False, logits_out=logits)

    if args.profile_steps:
        for s in range(args.profile_steps):
            step(s)
        torch.cuda.synchronize()
        return
    for s in range(max(3, args.warmup)):
        step(s)
    torch.cuda.synchronize()
    clk = ClockSampler(phys_index(local))
    t_end = time.time() + 2.0
    s = 0
    while time.time() < t_end:
        for _ in range(50):
            step(s)
            s += 1
        torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    # steps replayed from a CUDA graph of one pass over the pool (the three
    # launches of a step take less GPU time than Python takes to issue them)
    reps = max(1, args.steps // npool)
    ms = graph_ms_per_step(torch, step, npool, reps, stream)
    clocks = clk.stop()
    err, _ = ctx.status(reset=True)
    # the GEMM alone (the tensor-core kernel), the same way
    gemm_ms = graph_ms_per_step(torch, gemm, npool, reps, stream)
    eager_t0 = time.perf_counter()
    for s in range(args.steps):
        step(s)
    torch.cuda.synchronize()
    eager_ms = (time.perf_counter() - eager_t0) * 1e3 / args.steps
    flops = wl.head_flops(B, d, N)
    tf_peak, tf_kind = tensor_peaks()
    hbm_peak, hbm_kind = peaks()
    achieved = flops / (gemm_ms / 1e3) / 1e12
    gemm_bytes = wbytes + B * d * 2 + B * N * 4 + N * 4
    # e2e: hidden states from pinned host memory, ids back, through the public call
    hh = [torch.from_numpy(np.ascontiguousarray(pool[0]["h"].cpu().numpy())).pin_memory()]
    ids_h = torch.empty(B, dtype=torch.int32).pin_memory()
    hdev = torch.empty((B, d), dtype=torch.int16, device=dev)

    def hstep(s):
        hdev.copy_(hh[0], non_blocking=True)
        p = pool[s % npool]
        ctx.head_sample(hdev, p["W"], bias, gamma, beta, hist, off, params, rng, out_ids=ids, norm_out=norm,
                        logits_out=logits)
        ids_h.copy_(ids, non_blocking=True)

    for s in range(3):
        hstep(s)
    torch.cuda.synchronize()
    e0.record(stream)
    for s in range(args.steps):
        hstep(s)
    e1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1) / args.steps
    # CPU stand-in: float32 GEMM on the host (numpy BLAS, all threads) + the
    # C oracle's sampling on those logits, one step of the same batch
    cpu = None
    if not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as orc
        o = orc.Oracle()
        x = wl.bf16_float(hb.hidden)
        xm = x - x.mean(axis=1, keepdims=True)
        y = xm / np.sqrt((xm * xm).mean(axis=1, keepdims=True) + 1e-5) * hb.gamma + hb.beta
        Wf = wl.bf16_float(hb.weight)
        t0 = time.perf_counter()
        n = 0
        while True:
            lg = y.astype(np.float32) @ Wf.T + hb.bias
            o.sample_batch(np.ascontiguousarray(lg, np.float32), N, hb.hist, hb.hist_off, hb.params, hb.rng.copy(),
                           nthreads=os.cpu_count() or 1)
            n += 1
            if time.perf_counter() - t0 > min(args.cpu_seconds, 5.0):
                break
        el = time.perf_counter() - t0
        cpu = {"value": B * n / el, "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
               "sample": f"{n} steps of the config-3 batch: numpy float32 GEMM (multithreaded BLAS) + the C "
                         f"oracle's sampling on {os.cpu_count()} threads (the reference's head runs in MLX, "
                         "which is not installed)"}
    line = {
        "metric": "sampled tokens/s (LM head + sampling, B=256, d=1280, V=8194, config 3)",
        "value": B / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1, "steps": reps * npool, "warmup": args.warmup,
        "ms_per_step": ms, "eager_ms_per_step": eager_ms,
        "timing": "CUDA-graph replay of one pass over the weight pool; eager_ms_per_step: the same step "
                  "issued from Python each time (host-bound)",
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 GEMM (fp32 accumulate) + f32/f64 sampling", "data": "synthetic",
        "config": {"workload": "config3: hidden bf16 N(0,1) [256,1280], head bf16 N(0,0.02^2) [8194,1280], "
                               "LayerNorm + bias, config-0 sampling, history 512",
                   "l2": f"pool of {npool} weight matrices rotated (> 2x L2)"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": tf_peak, "unit": "TFLOP/s",
                     "frac": achieved / tf_peak, "traffic": None, "kernel": "head_gemm_kernel",
                     "peak_kind": tf_kind, "flops_per_launch": flops, "gemm_ms": gemm_ms,
                     "hbm_achieved_gbs": gemm_bytes / (gemm_ms / 1e3) / 1e9, "hbm_peak": hbm_peak,
                     "hbm_frac": gemm_bytes / (gemm_ms / 1e3) / 1e9 / hbm_peak},
        "cpu_baseline": cpu,
        "e2e": {"value": B / (ms_e2e / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": B * d * 2,
                "d2h_bytes_per_step": B * 4, "ms_per_step": ms_e2e},
        "gpu_launches": 3 * args.steps,
        "clocks": clocks, "device_errors": err,
    }
    print(json.dumps(line), flush=True)
    ctx.close()


def run_qgemv(args):
    """Quantized decode projections (gpt2.cpp:52-73, int8 group 64: the
    reference's product default): per step the four projections of one GPT-2
    layer (c_attn 1280->3840, attn c_proj 1280->1280, mlp c_fc 1280->5120, mlp
    c_proj 5120->1280) at B=1, the weights of 12 layers rotating (> 2x L2)."""
    import torch

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    c4s = load_pkg()
    ctx = c4s.SamplingContext(max_vocab=64, device=0)
    stream = torch.cuda.current_stream(dev)
    D, bits, group, B = 1280, 8, 64, 1
    shapes = [(3 * D, D), (D, D), (4 * D, D), (D, 4 * D)]
    g = torch.Generator(device=dev).manual_seed(0)
    layers = []
    for _ in range(12):
        lay = []
        for N, K in shapes:
            w = torch.randn((N, K), device=dev, generator=g) * 0.02
            lay.append((*ctx.quantize_affine(w, group, bits), torch.zeros(N, device=dev), N, K))
            del w
        layers.append(lay)
    x = {K: torch.randn((B, K), device=dev, generator=g) for K in (D, 4 * D)}
    y = {N: torch.empty((B, N), device=dev) for N, _ in shapes}

    def step(s):
        for q, sc, bi, bo, N, K in layers[s % len(layers)]:
            ctx.qgemv(x[K], q, sc, bi, group, bits, bias_out=bo, out=y[N])

    if args.profile_steps:
        for s in range(args.profile_steps):
            step(s)
        torch.cuda.synchronize()
        return
    for s in range(max(3, args.warmup)):
        step(s)
    torch.cuda.synchronize()
    clk = ClockSampler(phys_index(0))
    t_end = time.time() + 2.0
    s = 0
    while time.time() < t_end:
        for _ in range(20):
            step(s)
            s += 1
        torch.cuda.synchronize()
    ms = graph_ms_per_step(torch, step, len(layers), max(1, args.steps // len(layers)), stream)
    clocks = clk.stop()
    wbytes = sum(N * K * (bits / 8 + 8 / group) for N, K in shapes)
    io_bytes = sum(4 * B * (N + K) + 4 * N for N, K in shapes)
    hbm_peak, kind = peaks()
    gbs = (wbytes + io_bytes) / (ms / 1e3) / 1e9
    line = {
        "metric": "quantized decode projections per GPT-2 layer (int8 group 64, B=1)", "value": ms * 1e3,
        "unit": "us per layer", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "timing": "CUDA-graph replay of the 12 layers' projections (4 launches per layer)",
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "int8 weights, f32 math",
        "data": "synthetic",
        "config": {"workload": "GPT-2 d=1280 layer: 1280x3840, 1280x1280, 1280x5120, 5120x1280, B=1",
                   "l2": "12 layers of weights rotated (266 MB > 2x L2)"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                     "traffic": None, "kernel": "qgemv_kernel", "peak_kind": kind,
                     "alg_bytes_per_step": wbytes + io_bytes},
        "gpu_launches": 4 * args.steps, "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    ctx.close()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "c4":
        run_vocab_sharded(args)
    elif args.workload == "c3":
        run_head(args)
    elif args.workload == "qgemv":
        run_qgemv(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
