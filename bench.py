#!/usr/bin/env python
"""Benchmark of the B200 streaming top-k SAE encoder (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config 2|3|4|5]

One step = one exact top-k encode of one batch (B rows) over all F features.
Default workload (the north-star target):
exact bf16, B=128, d=2048, F=262144, k=64, X ~ N(0,1), W_enc rows N(0,1)
scaled to unit L2 norm, b_enc ~ N(0, 0.01) (std 0.1); W_enc is 1 GiB, larger
than L2, so no L2 flush is needed between steps.  With N > 1 (torchrun, one
process per GPU) W_enc is sharded along F (streamtopk_sae.shard.ShardedEncoder,
strong scaling: total work fixed): each rank's score kernel selects its rows'
best k keys in its own tail and stores them into every rank's receive buffer
over NVLink (CUDA IPC peer stores, per-row step tags, bounded waits), then
merges the N lists of its rows: one kernel launch per step, replayed from a
CUDA graph.  When a rank cannot map its peers the lists travel by an NCCL
all-gather and a finish kernel instead (--transport nccl forces that).

Printed on rank 0: one JSON line with the contract's keys, plus
  roofline      the fused tcgen05 kernel's algorithmic bytes / its CUDA-event
                time (N=1: an instrumented re-run of the same K steps right
                after the un-instrumented timed region; N>1: event nodes in the
                timed graph), against the measured HBM copy bandwidth
                (MEASURED_PEAKS.json);
  cpu_baseline  the reference's own CPU op (compiled from its sources into
                oracle/_ref) on a bounded sample, rank 0 at N=1 only;
  e2e           the same metric through the public API with pinned host X in
                and host V/I out every step (by default the upload of step
                i+1 overlaps the kernels of step i on a copy stream);
  clocks        nvidia-smi samples taken during the timed region.
--impl reference times the reference's CPU implementation (oracle/_ref, all
host cores through a process pool) on the same metric.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "streamtopk-sae_b200"))

METRIC = "SAE encode rows/sec & % of HBM/tensor roofline at B,d,F,k; 1/2/4/8 B200"
CONFIGS = {
    2: dict(B=128, d=768, F=65536, k=32, dtype="bf16", w_init="normal_1_over_d", mode="exact"),
    3: dict(B=128, d=2048, F=262144, k=64, dtype="bf16", w_init="unit_rows", mode="exact"),
    4: dict(B=128, d=2048, F=1048576, k=32, dtype="bf16", w_init="unit_rows", mode="approx", c=32),
    5: dict(B=4096, d=4096, F=262144, k=128, dtype="fp16", w_init="normal_1_over_d", mode="exact"),
}
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def esize(dtype):
    return 4 if dtype == "fp32" else 2


def alg_bytes(B, d, F, k, dtype):
    if dtype == "fp8":   # bf16 X in, E4M3 W_enc, fp32 bias and per-feature scale, (B, k) out
        return B * d * 2 + F * d + 8 * F + 8 * B * k
    """Algorithmic bytes per encode (reference bench/run_bandwidth.py:73-78)."""
    return B * d * esize(dtype) + F * d * esize(dtype) + 4 * F + 8 * B * k


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), float(j.get("bf16_tflops_sustained", j["bf16_tflops"])), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, 1400.0, "fallback"


def profiled_traffic(config_id, n_gpus):
    """DRAM bytes per fused-kernel launch from the committed ncu summary, if any."""
    p = os.path.join(REPO, "profiles", f"fused_topk_kernel_cfg{config_id}.txt")
    try:
        for line in open(p):
            if line.startswith(f"traffic_bytes_per_launch_n{n_gpus}:"):
                return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


def float64_row_scores(X, W, b, rows, chunk=32768, w_scale=None):
    """float64 scores of the sampled rows over all features (on X's device);
    W's rows times w_scale when given (the fp8 path's dequantized W_enc)."""
    import torch
    Xs = X[rows].double()
    out = torch.empty((len(rows), W.shape[0]), dtype=torch.float64, device=X.device)
    for f0 in range(0, W.shape[0], chunk):
        f1 = min(W.shape[0], f0 + chunk)
        Wc = W[f0:f1].double()
        if w_scale is not None:
            Wc = Wc * w_scale[f0:f1, None].double()
        out[:, f0:f1] = Xs @ Wc.T + b[f0:f1].double()
    return out


def rows_match(V, I, S, k, rtol):
    """Tie-aware check of sampled output rows against their float64 scores S.

    Per row (v_k = k-th largest score, tau = rtol * max |top-k score|): sorted
    values within tau of the true top-k, distinct indices, every predicted index
    scoring >= v_k - tau, every index scoring > v_k + tau predicted, and each
    value within tau of the score at its index.
    """
    import torch
    for r in range(S.shape[0]):
        top, _ = torch.topk(S[r], k)
        vk = top[-1]
        tau = rtol * max(float(top.abs().max()), 1e-30)
        pv = V[r].double()
        idx = I[r].long()
        if int(idx.min()) < 0 or int(idx.max()) >= S.shape[1] or torch.unique(idx).numel() != k:
            return False
        si = S[r][idx]
        if float((torch.sort(pv, descending=True).values - top).abs().max()) > tau:
            return False
        if float((pv - si).abs().max()) > tau or bool((si < vk - tau).any()):
            return False
        must = torch.nonzero(S[r] > vk + tau).flatten()
        if must.numel() and not bool(torch.isin(must, idx).all()):
            return False
    return True


class ClockSampler:
    """nvidia-smi samples of one GPU while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, local_rank):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        self.gpu = vis.split(",")[local_rank] if vis else str(local_rank)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()
        return False

    def summary(self):
        rows = [r for r in csv.reader(io.StringIO(self.out)) if len(r) >= 9]
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except ValueError:
                continue
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU reference arm / baseline (the reference's own CPU op from oracle/_ref).
# ---------------------------------------------------------------------------

def _ref_worker_init():
    import torch
    torch.set_num_threads(1)
    sys.path.insert(0, REPO)
    from oracle import oracle
    oracle._ref_mod()


def _ref_worker(args):
    X, W, b, k = args
    from oracle import oracle
    oracle.ref_cpu_topk(X, W, b, k)
    return X.shape[0]


def reference_inputs(cfg, f_sample, seed=0):
    """fp32 CPU inputs with the config's distributions, F cut to f_sample."""
    import torch
    g = torch.Generator()
    g.manual_seed(seed)
    dt = torch.bfloat16 if cfg["dtype"] == "bf16" else (torch.float16 if cfg["dtype"] == "fp16" else torch.float32)
    X = torch.randn(cfg["B"], cfg["d"], generator=g).to(dt).float()
    W = torch.randn(f_sample, cfg["d"], generator=g)
    if cfg["w_init"] == "unit_rows":
        W = W / W.norm(dim=1, keepdim=True).clamp_min(1e-8)
    else:
        W = W / cfg["d"] ** 0.5
    W = W.to(dt).float()
    b = torch.randn(f_sample, generator=g) * 0.1
    return X.contiguous(), W.contiguous(), b.contiguous()


def time_reference_single(cfg, budget_s=10.0):
    """1-thread reference CPU op on (all rows) x (F sample); rows/s scaled to full F."""
    sys.path.insert(0, REPO)
    from oracle import oracle
    if not oracle.ref_available():
        return None
    k = cfg["k"]
    calib_f = 2048
    X, W, b = reference_inputs(cfg, calib_f)
    t0 = time.perf_counter()
    oracle.ref_cpu_topk(X, W, b, k)
    per_feature = (time.perf_counter() - t0) / calib_f
    f_s = int(min(cfg["F"], max(4096, (budget_s / 3) / per_feature)) // 512 * 512)
    X, W, b = reference_inputs(cfg, f_s)
    oracle.ref_cpu_topk(X, W, b, k)
    ts = []
    for _ in range(3):
        t0 = time.perf_counter()
        oracle.ref_cpu_topk(X, W, b, k)
        ts.append(time.perf_counter() - t0)
    t = statistics.median(ts)
    rows_s = cfg["B"] / t * (f_s / cfg["F"])
    return {"value": rows_s, "unit": "rows/s", "cores": 1, "kind": "reference",
            "extrapolated": {"measured_F": f_s, "reported_F": cfg["F"], "how": "x F_sample/F (linear in F)"},
            "sample": f"reference topk_sae_cpu (oracle/_ref, 1 thread as shipped: no OpenMP) on all "
                      f"{cfg['B']} rows x {f_s} of {cfg['F']} features, fp32 upcast, median of 3; "
                      f"rows/s scaled by F_sample/F (cost is linear in F); host has {os.cpu_count()} cores"}


def run_reference(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    sys.path.insert(0, REPO)
    from oracle import oracle
    if not oracle.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref not built (python oracle/build_ref.py)"}))
        return 0
    import torch
    import torch.multiprocessing as mp
    procs = max(1, min(os.cpu_count() or 1, cfg["B"]))
    # Size each step so that warmup + steps take about a minute in total.
    X, W, b = reference_inputs(cfg, 2048)
    t0 = time.perf_counter()
    oracle.ref_cpu_topk(X, W, b, cfg["k"])
    per_feature_all_rows = (time.perf_counter() - t0) / 2048
    total_budget = 60.0
    step_budget = total_budget / max(1, args.steps + args.warmup)
    f_s = int(step_budget * procs / per_feature_all_rows)
    f_s = max(512, min(cfg["F"], f_s // 512 * 512))
    X, W, b = reference_inputs(cfg, f_s)
    W.share_memory_()
    X.share_memory_()
    b.share_memory_()
    bounds = [cfg["B"] * i // procs for i in range(procs + 1)]
    work = [(X[bounds[i]:bounds[i + 1]], W, b, cfg["k"]) for i in range(procs) if bounds[i + 1] > bounds[i]]
    ctx = mp.get_context("spawn")
    with ctx.Pool(len(work), initializer=_ref_worker_init) as pool:
        for _ in range(args.warmup):
            pool.map(_ref_worker, work)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            pool.map(_ref_worker, work)
        el = time.perf_counter() - t0
    ms_step = el / args.steps * 1e3
    value = cfg["B"] / (el / args.steps) * (f_s / cfg["F"])
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": config_dict(args, cfg),
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": len(work), "kind": "reference",
                         "sample": f"reference topk_sae_cpu (compiled from its sources into oracle/_ref) in "
                                   f"{len(work)} spawned processes, each on a row shard, all {cfg['B']} rows x "
                                   f"{f_s} of {cfg['F']} features per step (fp32 upcast); rows/s scaled by "
                                   f"F_sample/F (cost is linear in F)"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "extrapolated": {"measured_F": f_s, "reported_F": cfg["F"],
                         "how": "rows/s on an F sample x F_sample/F (the CPU op's cost is linear in F)"},
    }
    print(json.dumps(line))
    return 0


def config_dict(args, cfg):
    tag = f"cfg{args.config}" + (" (shape override)" if args.shape else "")
    d = {"workload": (f"{tag}: {cfg['mode']} {cfg['dtype']} B={cfg['B']} d={cfg['d']} F={cfg['F']} "
                      f"k={cfg['k']}" + (f" c={cfg['c']}" if cfg["mode"] == "approx" else "") +
                      (f", W_enc F-sharded over {args.gpus} GPUs" if args.gpus > 1 else "")),
         "B": cfg["B"], "d": cfg["d"], "F": cfg["F"], "k": cfg["k"], "global_batch": cfg["B"],
         "parallelism": f"F-shard{args.gpus}" if args.gpus > 1 else "single-gpu",
         "l2": "inputs larger than L2: each rank streams >= 128 MiB of W_enc per step"}
    if cfg["dtype"] == "fp8":
        d["fp8"] = ("E4M3 W_enc with one fp32 scale per feature (quantized once); X bf16, quantized per row to E4M3 "
                    "on every call; kind::f8f6f4 with fp32 accumulation (an extension: lossy, reported as recall)")
    return d


# ---------------------------------------------------------------------------
# B200 arm.
# ---------------------------------------------------------------------------

def run_b200(args, cfg):
    import torch
    import torch.distributed as dist
    import streamtopk_sae as stk
    from streamtopk_sae import _capi
    from streamtopk_sae import shard as stk_shard

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    B, d, F, k = cfg["B"], cfg["d"], cfg["F"], cfg["k"]
    fp8 = cfg["dtype"] == "fp8"
    if fp8 and (world > 1 or cfg["mode"] != "exact"):
        raise SystemExit("--dtype fp8: the exact encode on one GPU")
    dtype = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32, "fp8": torch.bfloat16}[cfg["dtype"]]
    X, W, b = stk.make_inputs(B, d, F, dtype=dtype, seed=0, device=dev, w_init=cfg["w_init"])
    f0, f1 = stk_shard.shard_bounds(F, world, rank)
    # Correctness of what is timed (outside the timed region): float64 scores of
    # a few rows over all F, and at N > 1 the single-GPU encode of the full
    # W_enc on rank 0 (every rank holds the full W_enc before slicing).
    check_rows = sorted({0, B // 3, (2 * B) // 3, B - 1})
    bf16_exact = None
    if fp8:
        # E4M3 W_enc (one scale per feature) and X quantized per row on every
        # call: parity is against float64 scores of the quantized operands,
        # and recall against the bf16 exact encode measures the quantization.
        from streamtopk_sae import fp8 as stk_fp8
        W8, w_scale = stk_fp8.quantize_weights(W)
        Q, sx = stk_fp8.quantize_rows(X)
        S_rows = float64_row_scores(Q.float() * sx[:, None], W8, b, check_rows, w_scale=w_scale)
        bf16_exact = stk.topk_sae_cuda_exact(X, W, b, k)
        torch.cuda.synchronize(dev)
        del W, Q, sx
        W = None
        torch.cuda.empty_cache()
    else:
        S_rows = float64_row_scores(X, W, b, check_rows) if rank == 0 else None
    single_gpu = None
    if world > 1 and rank == 0:
        single_gpu = stk.topk_sae_cuda_exact(X, W, b, k)
        torch.cuda.synchronize(dev)
    if world > 1:
        W = W[f0:f1].clone()
        b = b[f0:f1].clone()
        torch.cuda.empty_cache()
        enc = stk_shard.ShardedEncoder(W, b, F, f0, k, mode=cfg["mode"], c=cfg.get("c"),
                                       transport=args.transport, max_rows=B)
        step = enc.encode
    elif fp8:
        step = lambda x: stk_fp8.topk_sae_cuda_exact_fp8(x, W8, w_scale, b, k)  # noqa: E731
    elif cfg["mode"] == "approx":
        step = lambda x: stk.topk_sae_cuda_approx(x, W, b, k, cfg["c"])  # noqa: E731
    else:
        step = lambda x: stk.topk_sae_cuda_exact(x, W, b, k)  # noqa: E731
    # Steps of the timed loop: the pipelined encode where it applies (each
    # batch finished by the next batch's score kernel, the last by flush()),
    # else one call per batch.  deferred: a batch's V/I are complete only after
    # the next submit / flush.
    pipe = None
    flush = lambda: None  # noqa: E731
    submit, deferred = step, False
    if world > 1:
        submit, flush, deferred = enc.submit, enc.flush, True
    elif not fp8 and cfg["mode"] == "exact" and not args.no_pipeline:
        pipe = stk.EncodePipeline(B, d, F, k, dtype, device=dev)
        submit = lambda x: pipe.submit(x, W, b)  # noqa: E731
        flush, deferred = pipe.flush, True

    stream = torch.cuda.current_stream(dev)
    from streamtopk_sae.graph import CapturedEncode

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for _ in range(max(args.warmup, 3)):
        submit(X)
    flush()
    torch.cuda.synchronize(dev)
    assert _capi.device_error(stream.cuda_stream) == 0

    # ---------------- timed region (device-resident inputs)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    if world == 1:
        # One GPU: the host enqueues a step far faster than the GPU runs it, so
        # steps are launched eagerly.  The timed region is un-instrumented (the
        # library's per-kernel events would sit between the score kernel and
        # its programmatically-dependent merge and cost ~10 us per step); the
        # same K steps are then run again with CUDA events around every library
        # kernel to get the kernel durations and launch counts.
        G = 1
        barrier()
        torch.cuda.synchronize(dev)
        with ClockSampler(local) as clk:
            e0.record(stream)
            for _ in range(args.steps):
                submit(X)
            flush()
            e1.record(stream)
            torch.cuda.synchronize(dev)
        el_ms = e0.elapsed_time(e1)
        with _capi.KernelTimer(max_launches=args.steps * 4 + 16) as kt:
            for _ in range(args.steps):
                submit(X)
            flush()
            torch.cuda.synchronize(dev)
        launches = sum(kt.launches.values())
    else:
        # N GPUs: per-rank GPU time per step is small enough that host launch
        # work (checks, ctypes, NCCL enqueue) would dominate, so each timed
        # iteration replays a CUDA graph of G encode steps (memset, kernels and
        # the peer-store exchange, or the NCCL all-gather), as a serving loop
        # would.
        # The timed graph holds no profiling events (they would sit between
        # programmatically dependent kernels); a second, instrumented graph of
        # the same G steps gives the per-kernel durations afterwards.
        G = next(g for g in (8, 4, 2, 1) if args.steps % g == 0)
        timed = CapturedEncode(submit, X, steps=G, warmup=0, finish=flush)
        barrier()
        torch.cuda.synchronize(dev)
        with ClockSampler(local) as clk:
            e0.record(stream)
            for _ in range(args.steps // G):
                timed.replay()
            e1.record(stream)
            torch.cuda.synchronize(dev)
        barrier()
        el_ms = e0.elapsed_time(e1)
        timed.close()
        del timed
        with _capi.KernelTimer(max_launches=G * 4 + 16) as kt:
            inst = CapturedEncode(submit, X, steps=G, warmup=0, finish=flush)   # event nodes around each kernel
            barrier()
            for _ in range(4):
                inst.replay()
            torch.cuda.synchronize(dev)
            barrier()
            inst.close()
            del inst
        # kt holds the G steps of the last replay (event nodes re-record per replay)
        launches = sum(kt.launches.values()) // G * args.steps
    assert _capi.device_error(stream.cuda_stream) == 0
    t = torch.tensor([el_ms], device=dev, dtype=torch.float64)
    fused_ms = kt.ms["fused_topk_kernel"] + kt.ms["simt_topk_kernel"]
    fused_n = kt.launches["fused_topk_kernel"] + kt.launches["simt_topk_kernel"]
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    el_ms = float(t.item())
    value = B * args.steps / (el_ms / 1e3)

    # ---------------- parity of the timed step (one more, untimed, call on every rank)
    Vp, Ip = submit(X)
    flush()
    torch.cuda.synchronize(dev)
    parity = None
    if rank == 0:
        rtol = 1e-5 if cfg["dtype"] == "fp32" else 1e-3
        parity = {"rows_vs_float64": rows_match(Vp[check_rows].cpu(), Ip[check_rows].cpu(), S_rows.cpu(), k, rtol),
                  "rows_checked": len(check_rows), "rtol": rtol}
        if single_gpu is not None:
            parity["bitwise_vs_single_gpu"] = bool(torch.equal(Vp, single_gpu[0]) and torch.equal(Ip, single_gpu[1]))
        if bf16_exact is not None:
            parity["float64_of"] = "the quantized operands (x_scale * X8, w_scale * W8)"
            parity["recall_vs_bf16_exact"] = stk.recall_at_k(Ip.long(), bf16_exact[1].long())
        parity["ok"] = all(v for kk, v in parity.items() if kk in ("rows_vs_float64", "bitwise_vs_single_gpu"))
        S_rows = single_gpu = None
    del Vp, Ip

    # ---------------- end to end through the public API, host buffers
    Xh = X.cpu().pin_memory()
    Vh = torch.empty((B, k), dtype=torch.float32).pin_memory()
    Ih = torch.empty((B, k), dtype=torch.int32).pin_memory()
    e2e_steps = max(1, min(args.steps, 2000))
    overlap = not args.e2e_serial
    graphs = []
    if world == 1:
        # The public API called eagerly on a device buffer (two when overlapped):
        # the pipelined encode (or the one-call op where it does not apply).
        Xd2 = [torch.empty_like(X) for _ in range(2 if overlap else 1)]
        runs = [(lambda xd: (lambda: submit(xd)))(xd) for xd in Xd2]
        e2e_deferred = deferred
    else:
        # One CUDA graph of one encode step per input buffer (graph.CapturedEncode:
        # its static X is the buffer the host copy lands in).
        graphs = [CapturedEncode(step, X, steps=1, warmup=1 if i == 0 else 0) for i in range(2 if overlap else 1)]
        Xd2 = [g_.X for g_ in graphs]
        runs = [g_.replay for g_ in graphs]
        e2e_deferred = False

    if overlap:
        # A serving loop: X of step i+1 is uploaded on a copy stream while the
        # kernels of step i run (two device buffers); V/I come back on another.
        h2d = torch.cuda.Stream(device=dev)
        d2h = torch.cuda.Stream(device=dev)
        copied = [torch.cuda.Event(), torch.cuda.Event()]
        consumed = [torch.cuda.Event(), torch.cuda.Event()]
        readback = [torch.cuda.Event(), torch.cuda.Event()]
        flushed = torch.cuda.Event()

        def read_back(VI, after, slot):
            V, I = VI
            d2h.wait_event(after)
            with torch.cuda.stream(d2h):
                V.record_stream(d2h)
                I.record_stream(d2h)
                Vh.copy_(V, non_blocking=True)
                Ih.copy_(I, non_blocking=True)
                readback[slot].record(d2h)

        def e2e_run(n):
            h2d.wait_stream(stream)
            with torch.cuda.stream(h2d):
                Xd2[0].copy_(Xh, non_blocking=True)
                copied[0].record(h2d)
            pending = None
            for i in range(n):
                cur = i & 1
                if i + 1 < n:
                    nxt = cur ^ 1
                    with torch.cuda.stream(h2d):
                        h2d.wait_event(consumed[nxt])   # step i-1 is done reading that buffer
                        Xd2[nxt].copy_(Xh, non_blocking=True)
                        copied[nxt].record(h2d)
                stream.wait_event(copied[cur])
                if world > 1 and i >= 2:
                    stream.wait_event(readback[cur])  # V/I of this graph's previous replay are read
                V, I = runs[cur]()            # the public API / the captured ShardedEncoder.encode
                consumed[cur].record(stream)
                if e2e_deferred:
                    # Pipelined: step i-1's rows were finished by step i's launch.
                    if pending is not None:
                        read_back(pending, consumed[cur], cur)
                    pending = (V, I)
                else:
                    read_back((V, I), consumed[cur], cur)
            if pending is not None:
                flush()
                flushed.record(stream)
                read_back(pending, flushed, 0)
            stream.wait_stream(d2h)
    else:
        def e2e_run(n):
            for _ in range(n):
                Xd2[0].copy_(Xh, non_blocking=True)
                V, I = runs[0]()
                if e2e_deferred:
                    flush()
                Vh.copy_(V, non_blocking=True)
                Ih.copy_(I, non_blocking=True)

    e2e_run(3)
    torch.cuda.synchronize(dev)
    barrier()
    e0.record(stream)
    e2e_run(e2e_steps)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    t2 = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t2, op=dist.ReduceOp.MAX)
    e2e_value = B * e2e_steps / (float(t2.item()) / 1e3)
    for g_ in graphs:
        g_.close()
    graphs = runs = Xd2 = None
    torch.cuda.synchronize(dev)

    # ---------------- roofline of the dominant kernel (this rank's shard)
    hbm, tf, tf_sus, src = load_peaks()
    Fs = f1 - f0
    fused_avg_ms = fused_ms / max(fused_n, 1)
    if cfg["mode"] != "exact" or cfg["B"] <= 256:
        per_launch = alg_bytes(B, d, Fs, k, cfg["dtype"])
        achieved = per_launch / (fused_avg_ms / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "traffic": (None if args.shape or cfg["dtype"] == "fp8" else profiled_traffic(args.config, world)),
                "kernel": "fused_topk_kernel", "kernel_ms": fused_avg_ms,
                "algorithmic_bytes_per_launch": per_launch,
                "peak_source": f"{src} (MEASURED_PEAKS.json hbm_gbs)" if src == "measured" else "fallback"}
    else:
        flops = 2.0 * B * d * Fs
        achieved = flops / (fused_avg_ms / 1e3) / 1e12
        peak = tf_sus
        roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "traffic": (None if args.shape or cfg["dtype"] == "fp8" else profiled_traffic(args.config, world)), "kernel": "fused_topk_kernel",
                "kernel_ms": fused_avg_ms, "algorithmic_flops_per_launch": flops,
                "peak_source": f"{src} bf16_tflops_sustained (fp16 assumed equal)"}

    line = None
    if rank == 0:
        cpu = time_reference_single(cfg) if world == 1 and not args.no_cpu_baseline else None
        line = {
            "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": el_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": cfg["dtype"],
            "data": "synthetic (seeded Gaussian, BASELINE.json distributions)",
            "config": config_dict(args, cfg), "roofline": roof, "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "rows/s", "h2d_bytes_per_step": Xh.numel() * Xh.element_size() * world,
                    "d2h_bytes_per_step": (Vh.numel() * 4 + Ih.numel() * 4) * world,
                    "path": (((("streamtopk_sae.EncodePipeline.submit (each batch finished by the next batch's launch)"
                                if deferred else "streamtopk_sae.topk_sae_cuda_exact")) if world == 1 else
                              "streamtopk_sae.shard.ShardedEncoder.encode in CUDA graphs (graph.CapturedEncode)") +
                             (", X of step i+1 uploaded on a copy stream during step i, V/I read back on another"
                              if overlap else ", copies and kernels serialised on one stream"))},
            "parity": parity,
            "gpu_launches": launches, "graph_steps": G, "clocks": clk.summary(),
            "timed_api": ("ShardedEncoder.submit x G + flush, CUDA graph" if world > 1 else
                          "EncodePipeline.submit x K + flush" if deferred else "one call per step"),
            "exchange": (None if world == 1 else
                         "direct peer stores over NVLink (stk_exchange_*)" if enc.transport in ("p2p", "auto") else
                         "NCCL all_gather_into_tensor + merge kernel" +
                         (f" (p2p unavailable: {enc.fallback_reason})" if enc.fallback_reason else "")),
            "kernel_ms_per_step": {kk: v / (args.steps if world == 1 else G) for kk, v in kt.ms.items()},
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        enc.close()      # collective: unmaps the peers' exchange buffers
        barrier()
        torch.cuda.synchronize(dev)
        sys.stdout.flush()
        sys.stderr.flush()
        # Every graph holding NCCL work is released above; still, end the rank
        # without the NCCL teardown so a stuck communicator can never keep the
        # process (and its GPU) alive after the result is printed.
        os._exit(0)
    return 0


# ---------------------------------------------------------------------------
# Memory mode: the reference's working-memory and max-F benchmarks
# (bench/run_memory.py:40-70, bench/run_max_F.py:29-60 in the reference), each
# cell measured in a fresh subprocess so the caching allocator starts clean.
# ---------------------------------------------------------------------------
MEMORY_CELLS = [dict(CONFIGS[2], dtype="bf16"), dict(CONFIGS[2], dtype="fp16"), dict(CONFIGS[2], dtype="fp32"),
                CONFIGS[3], CONFIGS[4], CONFIGS[5]]
MAX_F_CONFIGS = [dict(B=128, d=768, k=32, dtype="bf16"), dict(B=2048, d=768, k=32, dtype="bf16"),
                 dict(B=128, d=2048, k=64, dtype="bf16")]   # the reference's two, plus the north-star shape


def _memory_cell(mode, B, d, F, k, dtype, c):
    """One cell in this (fresh) process: peak device memory of one call minus
    inputs and outputs = the call's working memory (the library's workspace)."""
    import torch
    import streamtopk_sae as stk
    dt = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[dtype]
    try:
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats()
        X, W, b = stk.make_inputs(B, d, F, dtype=dt, seed=0, device="cuda")
        torch.cuda.synchronize()
        base = torch.cuda.memory_allocated()   # the inputs (generation temporaries are freed)
        torch.cuda.reset_peak_memory_stats()
        if mode == "approx":
            V, I = stk.topk_sae_cuda_approx(X, W, b, k, c)
        else:
            V, I = stk.topk_sae_cuda_exact(X, W, b, k)
        torch.cuda.synchronize()
        peak = torch.cuda.max_memory_allocated()
        out = B * k * 8
        return {"status": "ok", "baseline_mem_mb": base / 1e6, "peak_mem_mb": peak / 1e6,
                "working_mem_mb": (peak - base - out) / 1e6}
    except torch.cuda.OutOfMemoryError:
        return {"status": "OOM"}


def _run_cell(mode, B, d, F, k, dtype, c=0, timeout=600):
    cmd = [sys.executable, os.path.abspath(__file__), "--_memory-cell", mode, str(B), str(d), str(F), str(k), dtype,
           str(c)]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, cwd=REPO)
    except subprocess.TimeoutExpired:
        return {"status": "TIMEOUT"}
    if r.returncode != 0:
        return {"status": "ERR:" + r.stderr.strip()[-300:]}
    return json.loads(r.stdout.strip().splitlines()[-1])


def run_memory(args):
    """Working memory per BASELINE config and the largest F (powers of two)
    that fits one GPU, one JSON line each."""
    for cfg in MEMORY_CELLS:
        res = _run_cell(cfg["mode"], cfg["B"], cfg["d"], cfg["F"], cfg["k"], cfg["dtype"], cfg.get("c", 0))
        print(json.dumps({"kind": "working_memory", **{kk: cfg[kk] for kk in ("mode", "B", "d", "F", "k", "dtype")},
                          "c": cfg.get("c"), **res}), flush=True)
    for cfg in MAX_F_CONFIGS:
        lo, hi, best = 14, 30, None
        while lo <= hi:
            mid = (lo + hi) // 2
            res = _run_cell("exact", cfg["B"], cfg["d"], 1 << mid, cfg["k"], cfg["dtype"])
            if res.get("status") == "ok":
                best, lo = 1 << mid, mid + 1
            else:
                hi = mid - 1
        print(json.dumps({"kind": "max_F", **cfg, "max_F": best, "search": "powers of two 2^14..2^30, "
                          "binary search, one subprocess per probe (reference bench/run_max_F.py)"}), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", type=int, default=3, choices=sorted(CONFIGS))
    ap.add_argument("--dtype", default=None, choices=["bf16", "fp16", "fp32", "fp8"],
                    help="input dtype override (config 2 is a dtype sweep); fp8: E4M3 W_enc with per-feature "
                         "scales and X quantized per row on every call (streamtopk_sae.fp8; N=1, exact)")
    ap.add_argument("--no-pipeline", action="store_true",
                    help="N=1: time the one-call op (topk_sae_cuda_exact) instead of the pipelined encode")
    ap.add_argument("--e2e-serial", action="store_true",
                    help="e2e: serialise each step's copies and kernels on one stream (default: the X upload "
                         "of step i+1 overlaps the kernels of step i on a copy stream)")
    ap.add_argument("--no-cpu-baseline", action="store_true",
                    help="omit the timed CPU sample (profiling runs)")
    ap.add_argument("--transport", default="auto", choices=["auto", "p2p", "nccl"],
                    help="N>1: cross-GPU exchange of the per-rank key lists (auto: p2p, NCCL if the "
                         "peer mappings cannot be set up)")
    ap.add_argument("--shape", default=None,
                    help="B,d,F,k override of the config's shape (small cases for ncu captures)")
    ap.add_argument("--memory", action="store_true",
                    help="working memory per BASELINE config and the largest F per GPU (reference run_memory / "
                         "run_max_F), one JSON line each")
    ap.add_argument("--_memory-cell", nargs=7, default=None, help=argparse.SUPPRESS)
    args = ap.parse_args()
    if args._memory_cell:
        m, B, d, F, k, dt, c = args._memory_cell
        sys.path.insert(0, os.path.join(REPO, "streamtopk-sae_b200"))
        print(json.dumps(_memory_cell(m, int(B), int(d), int(F), int(k), dt, int(c))))
        return 0
    if args.memory:
        return run_memory(args)
    cfg = dict(CONFIGS[args.config])
    if args.shape:
        cfg["B"], cfg["d"], cfg["F"], cfg["k"] = (int(v) for v in args.shape.split(","))
    if args.dtype:
        cfg["dtype"] = args.dtype
    if args.impl == "reference":
        return run_reference(args, cfg)
    return run_b200(args, cfg)


if __name__ == "__main__":
    sys.exit(main())
