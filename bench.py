#!/usr/bin/env python
"""Mamba-2 SSD prefill benchmark on B200 (tokens/s, fraction of roofline).

    python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference]
                    [--workload nemotron|zamba2|long|decode|proj|...]

One step is one fused mixer-core prefill (conv1d+SiLU -> discretise ->
chunked SSD scan -> D skip, plus the conv-cache roll) over one batch of
synthetic inputs of the Nemotron-H-8B layer shape (B=4, L=8192, 128 heads x
64, d_state 128, 8 groups), already resident in HBM.  With N GPUs (torchrun,
one process per GPU) the 8 head-groups are split across ranks (8/N groups per
GPU, no collective in the path): total work is fixed ("strong" scaling) and
``value`` = B*L tokens / max-over-ranks step time.

The timed steps replay one captured CUDA graph per rotating input set (the
same library launches as an eager call, counted while capturing), bracketed
by a barrier and a synchronize, timed with CUDA events, max over ranks.  The
default run also reports ``sub_results``: the Zamba2 layer, the 131k-token
sequence (with the y all-gather when N > 1) and 64 decode steps at batch 256,
each at its own shape and sharded over the same ranks.

Rank 0 prints one JSON line.  ``e2e`` is the same metric through the public
API for host-resident activations (``alloy_b200.mixer.ssd_combined_streamed``):
the host->device copies of the step's inputs from pinned memory and the
device->host copies of its outputs happen inside the timed region, overlapped
piece by piece with the kernels.  ``--impl reference`` times the reference algorithm on the host
CPU (the numpy restatement in ``oracle/``; alloy's own MLX path cannot run on
this machine) on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import faulthandler
import json
import math
import os
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "Mamba-2 SSD prefill tokens/s (Nemotron-H shape) at 1/2/4/8 B200; % roofline"

WORKLOADS = {
    "nemotron": dict(name="nemotron_h_8b_mamba2_layer_prefill", B=4, L=8192, H=128, P=64, N=128,
                     G=8, K=4, Q=256),
    "zamba2": dict(name="zamba2_1.2b_mamba2_layer_prefill", B=8, L=4096, H=64, P=64, N=64, G=1,
                   K=4, Q=256),
    "long": dict(name="zamba2_1.2b_mamba2_layer_prefill_131k", B=1, L=131072, H=64, P=64, N=64,
                 G=1, K=4, Q=512),
    "decode": dict(name="nemotron_h_8b_mamba2_decode_step", B=256, L=1, H=128, P=64, N=128, G=8,
                   K=4, Q=256),
    # the gate and inner RMS norm after the scan (d_inner = H * P), full-width norm
    "gated_norm": dict(name="nemotron_h_8b_mamba2_gated_rmsnorm", B=4, L=8192, H=128, P=64,
                       N=128, G=8, K=4, Q=256),
    # the standalone conv1d + SiLU (split mode, alloy_conv1d_silu) over the layer's xBC
    "conv": dict(name="nemotron_h_8b_mamba2_conv1d_silu", B=4, L=8192, H=128, P=64, N=128, G=8,
                 K=4, Q=256),
    # backward of conv1d + SiLU over the layer's xBC (training: the reference's custom VJP)
    "conv_bwd": dict(name="nemotron_h_8b_mamba2_conv1d_silu_backward", B=4, L=8192, H=128, P=64,
                     N=128, G=8, K=4, Q=256),
    # the scan's backward (training) at the Zamba2 layer shape, fp32
    "scan_bwd": dict(name="zamba2_1.2b_mamba2_selective_scan_backward", B=8, L=4096, H=64, P=64,
                     N=64, G=1, K=4, Q=256),
    # the same with bf16 activations: the gradient scans on the tcgen05 scan
    "scan_bwd_bf16": dict(name="zamba2_1.2b_mamba2_selective_scan_backward_bf16", B=8, L=4096, H=64,
                          P=64, N=64, G=1, K=4, Q=256, dtype="bf16"),
    # the layer's in_proj and out_proj over the prefill's tokens (d_model 4096, d_inner 8192)
    "proj": dict(name="nemotron_h_8b_mamba2_projections_prefill", B=4, L=8192, H=128, P=64, N=128,
                 G=8, K=4, Q=256, d_model=4096),
    # one whole Mamba layer (projections, cached step, gate + norm) decoding at batch 1
    "decode_block": dict(name="nemotron_h_8b_mamba2_layer_decode_b1", B=1, L=64, H=128, P=64,
                         N=128, G=8, K=4, Q=256),
}

L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0

# DRAM bytes (read + write) of one prefill step on one GPU, measured with ncu
# over the step's three launches (B/C pre-pass, SSD, conv-cache roll), keyed by
# (workload, n_gpus); the capture's summary is kept under profiles/.
# Configurations not captured report None.
NCU_TRAFFIC_BYTES = {("nemotron", 1): (134.6 + 80.7 + 685.6 + 507.7 + 0.4) * 1e6,
                     ("long", 1): (33.6 + 0.3 + 830.7 + 1.3 + 1143.2 + 1028.0 + 0.1) * 1e6}


def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def measured_tensor_peak(sustained):
    """Dense bf16 TFLOP/s: the measured cuBLAS figure (burst, or sustained for
    kernels timed inside a long loop), else the fallback."""
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    key = "bf16_tflops_sustained" if sustained else "bf16_tflops"
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d[key]), f"measured {key}"
    except Exception:
        return (1400.0 if sustained else 1590.0), f"fallback {key}"


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while running."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x2: "applications_clocks_setting", 0x1: "gpu_idle", 0x10: "sync_boost"}

    def __init__(self, torch_device):
        self.samples = []
        self.ok = False
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            handle = nvml_handle(torch_device)
            if handle is None:
                handle = pynvml.nvmlDeviceGetHandleByIndex(torch_device)
            self.h = handle
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # pragma: no cover - no NVML
            self.err = str(e)

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                rs = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                try:
                    rs = self.nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
                except Exception:
                    rs = 0
            self.samples.append((time.perf_counter(), mhz, rs))
            time.sleep(0.005)

    def start(self):
        if self.ok:
            self.th = threading.Thread(target=self._run, daemon=True)
            self.th.start()

    def stop(self):
        if self.ok:
            self._stop.set()
            self.th.join()

    def summary(self, t0, t1):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": "nvml unavailable"}
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        if not inside and self.samples:
            mid = 0.5 * (t0 + t1)
            inside = [min(self.samples, key=lambda s: abs(s[0] - mid))]
        mhz = sorted(s[1] for s in inside)
        bits = 0
        for s in inside:
            bits |= s[2]
        reasons = sorted({name for b, name in self.REASONS.items() if bits & b} - {"gpu_idle"})
        return {"sm_mhz": mhz[len(mhz) // 2] if mhz else None, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(inside)}


# ------------------------------------------------------------------------ distributed
def dist_setup(gpus):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != gpus:
        raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={world}")
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def dist_max(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def local_problem(w, world, rank):
    """The shard of the layer this rank computes: (H_l, G_l) with heads split
    by head-group (or by heads inside the single group when G < world)."""
    H, G = w["H"], w["G"]
    if H % world:
        raise SystemExit(f"{H} heads do not split over {world} GPUs")
    if G % world == 0:
        return H // world, G // world
    if G == 1:
        return H // world, 1
    raise SystemExit(f"{G} groups do not split over {world} GPUs")


# ------------------------------------------------------------------------ our arm
def make_prefill_inputs(B, L, H, P, N, G, K, seed, device):
    """Synthetic inputs with the workload's distributions, generated on the GPU."""
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    conv_dim = H * P + 2 * G * N
    xBC = torch.randn((B, L, conv_dim), generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)
    dt_raw = torch.randn((B, L, H), generator=gen, device=device).to(torch.bfloat16)
    conv_w = torch.randn((conv_dim, K), generator=gen, device=device) * 0.5
    conv_b = torch.zeros(conv_dim, device=device)
    u = torch.exp(torch.empty(H, device=device).uniform_(math.log(1e-3), math.log(0.1), generator=gen))
    dt_bias = torch.log(torch.expm1(u))
    A_log = torch.empty(H, device=device).uniform_(0.0, math.log(16.0), generator=gen)
    D = torch.randn(H, generator=gen, device=device)
    return dict(xBC=xBC, dt_raw=dt_raw, conv_w=conv_w, conv_b=conv_b, dt_bias=dt_bias,
                A_log=A_log, D=D)


def prefill_problem(w, world, rank, dev, shard_of=None):
    """Inputs of this rank's share of a prefill workload: ``rot`` rotating
    input/output sets (each step reads and writes memory the previous steps
    did not touch, > 3x L2 in between), the call's keyword arguments and a
    ``step(i)`` that runs one fused prefill on set i % rot."""
    import torch
    from alloy_b200 import mixer

    H_l, G_l = local_problem(w, shard_of or world, rank)
    B, L, P, N, K, Q = w["B"], w["L"], w["P"], w["N"], w["K"], w["Q"]
    conv_dim = H_l * P + 2 * G_l * N
    kw = dict(n_heads=H_l, head_dim=P, d_state=N, n_groups=G_l, d_conv=K, chunk_size=Q)
    step_bytes = B * L * (conv_dim + H_l) * 2 + B * L * H_l * P * 2
    rot = max(1, math.ceil(3 * L2_BYTES / step_bytes))
    sets = []
    for r in range(rot):
        inp = make_prefill_inputs(B, L, H_l, P, N, G_l, K, seed=1000 * rank + r, device=dev)
        out = dict(y=torch.empty((B, L, H_l, P), dtype=torch.bfloat16, device=dev),
                   h=torch.empty((B, H_l, N, P), dtype=torch.float32, device=dev),
                   cs=torch.empty((B, K - 1, conv_dim), dtype=torch.bfloat16, device=dev))
        sets.append((inp, out))

    def step(i):
        inp, out = sets[i % rot]
        mixer.ssd_combined(inp["xBC"], inp["dt_raw"], inp["conv_w"], inp["conv_b"],
                           inp["dt_bias"], inp["A_log"], inp["D"], out=out["y"],
                           ssm_state_out=out["h"], conv_state_out=out["cs"], **kw)

    # algorithmic bytes of one step of this rank (one pass over the data)
    alg = (B * L * conv_dim * 2 + B * L * H_l * 2 + B * L * H_l * P * 2 + B * H_l * N * P * 4
           + B * (K - 1) * conv_dim * 2)
    return dict(H_l=H_l, G_l=G_l, kw=kw, rot=rot, sets=sets, step=step, alg=alg,
                step_bytes=step_bytes, tokens=B * L)


def graph_steps(pb, dev):
    """One CUDA graph per rotating input set, each holding one captured step
    (the library's launches of one fused prefill), so the timed loop replays
    them without host launch overhead between the kernels.  Returns the
    replaying step function and the library launches one step makes."""
    import torch
    from alloy_b200 import _lib
    lib = _lib.load()
    graphs = []
    per_step = 0
    for k in range(pb["rot"]):
        g = torch.cuda.CUDAGraph()
        n0 = lib.alloy_kernel_launch_count()
        with torch.cuda.graph(g):
            pb["step"](k)
        per_step = lib.alloy_kernel_launch_count() - n0
        graphs.append(g)
    torch.cuda.synchronize(dev)

    def replay(i):
        graphs[i % len(graphs)].replay()

    return replay, per_step, graphs


def time_steps(step, steps, warmup, world, stream, per_step_events=True):
    """Device time of ``steps`` calls of step(i) after ``warmup`` untimed ones,
    bracketed by a barrier and a synchronize on both sides: (ms per step over
    the whole region, ms per step summed over the per-step event pairs,
    library kernel launches in the region); times are local to this rank."""
    import torch
    from alloy_b200 import _lib
    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ks = [torch.cuda.Event(enable_timing=True) for _ in range(steps)] if per_step_events else []
    ke = [torch.cuda.Event(enable_timing=True) for _ in range(steps)] if per_step_events else []
    barrier(world)
    torch.cuda.synchronize()
    launches0 = _lib.load().alloy_kernel_launch_count()
    ev0.record(stream)
    for i in range(steps):
        if ks:
            ks[i].record(stream)
        step(i)
        if ke:
            ke[i].record(stream)
    ev1.record(stream)
    launches = _lib.load().alloy_kernel_launch_count() - launches0
    torch.cuda.synchronize()
    barrier(world)
    ms = ev0.elapsed_time(ev1) / steps
    kernel_ms = sum(a.elapsed_time(b) for a, b in zip(ks, ke)) / steps if ks else ms
    return ms, kernel_ms, launches


def sub_results(args, world, rank, dev, stream):
    """The other workloads, measured in the same run at their own shapes and
    sharded over the same ranks (heads for the one-group Zamba2 layers, batch
    rows for decode), each device-timed with CUDA events (max over ranks):
    the Zamba2-1.2B layer prefill, the 131,072-token Zamba2 sequence (with the
    all-gather of y as well when N > 1), and 64 decode steps at batch 256 of
    the Nemotron-H shape.  A few steps each, so the whole run stays short."""
    import torch
    peak, peak_kind = measured_peaks()
    res = {}
    steps, warm = max(5, min(args.steps, 20)), 3
    for key in ("zamba2", "long"):
        w = dict(WORKLOADS[key])
        pb = prefill_problem(w, world, rank, dev)
        for i in range(warm):
            pb["step"](i)
        replay, per_step, graphs = graph_steps(pb, dev)
        ms, kernel_ms, _ = time_steps(replay, steps, warm, world, stream)
        launches = per_step * steps
        del graphs
        ms, kernel_ms = dist_max(ms, world), dist_max(kernel_ms, world)
        gbs = pb["alg"] / (kernel_ms * 1e-3) / 1e9
        entry = {"value": pb["tokens"] / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms,
                 "steps": steps, "warmup": warm, "gpu_launches": launches,
                 "launch": "CUDA graph replay of one captured step per input set",
                 "config": {"batch": w["B"], "seq_len": w["L"], "n_heads": w["H"], "head_dim": w["P"],
                            "d_state": w["N"], "n_groups": w["G"], "chunk_size": w["Q"],
                            "shard": f"{pb['H_l']} heads / {pb['G_l']} groups per GPU",
                            "l2": f"{pb['rot']} rotating input/output sets of "
                                  f"{pb['step_bytes'] / 2**20:.0f} MiB"},
                 "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                              "frac": gbs / peak, "peak_source": f"{peak_kind} hbm_gbs",
                              "algorithmic_bytes_per_gpu": pb["alg"]}}
        if world > 1 and key == "long":
            entry["with_gather"] = run_with_gather(argparse.Namespace(steps=steps, warmup=warm),
                                                   pb["step"], pb["sets"], world, stream, pb["tokens"])
        res[w["name"]] = entry
        del pb
        torch.cuda.empty_cache()
    w = dict(WORKLOADS["decode"])
    dp = decode_problem(w, world, rank, dev)
    ms, _, launches = time_steps(dp["step"], 64, 4, world, stream, per_step_events=False)
    ms = dist_max(ms, world)
    gbs = dp["alg"] / (ms * 1e-3) / 1e9
    res[w["name"]] = {"value": gbs * world, "unit": "GB/s (whole job)", "ms_per_step": ms,
                      "tokens_per_s": w["B"] / (ms * 1e-3), "steps": 64, "warmup": 4,
                      "gpu_launches": launches,
                      "config": {"batch": w["B"], "batch_per_gpu": dp["B"], "n_heads": w["H"],
                                 "head_dim": w["P"], "d_state": w["N"], "n_groups": w["G"],
                                 "state_layout": "[B,H,P,N] f32", "conv_state_layout": "[B,C,K-1] bf16",
                                 "tokens_cycled": 64},
                      "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                                   "frac": gbs / peak, "peak_source": f"{peak_kind} hbm_gbs",
                                   "algorithmic_bytes_per_gpu": dp["alg"]}}
    del dp
    torch.cuda.empty_cache()
    return res


def run_ours(args, w):
    import torch
    from alloy_b200 import _lib, mixer

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local if world > 1 else 0)
    # --shard-of N on one GPU: the share of one rank of an N-GPU run (profiling)
    pb = prefill_problem(w, world, rank, dev,
                         shard_of=args.shard_of if world == 1 and args.shard_of else None)
    H_l, G_l, kw, rot, sets, step = pb["H_l"], pb["G_l"], pb["kw"], pb["rot"], pb["sets"], pb["step"]
    B, L, P, N, K, Q = w["B"], w["L"], w["P"], w["N"], w["K"], w["Q"]
    step_bytes = pb["step_bytes"]

    stream = torch.cuda.current_stream(dev)
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    # the timed steps replay one captured CUDA graph per input set (the same
    # launches as the eager call, without host launch gaps between kernels)
    replay, per_step, graphs = graph_steps(pb, dev)
    for i in range(2):
        replay(i)
    torch.cuda.synchronize()
    clocks = ClockSampler(dev.index)
    clocks.start()
    h0 = time.perf_counter()
    ms_local, kernel_ms_local, _ = time_steps(replay, args.steps, 0, world, stream)
    h1 = time.perf_counter()
    clocks.stop()
    launches = per_step * args.steps
    del graphs
    ms = dist_max(ms_local, world)
    kernel_ms = dist_max(kernel_ms_local, world)
    tokens = B * L
    value = tokens / (ms * 1e-3)

    alg = pb["alg"]
    peak, peak_kind = measured_peaks()
    achieved = alg / (kernel_ms_local * 1e-3) / 1e9
    achieved = dist_max(-achieved, world) * -1 if world > 1 else achieved  # slowest rank
    traffic = NCU_TRAFFIC_BYTES.get((args.workload, world))

    # ---- end to end through the public API, host buffers ----
    e2e = None if args.no_e2e else run_e2e(args, sets[0], kw, world, stream, B * L)
    # ---- the same steps followed by the all-gather of y (a caller that needs
    # every head of y on every GPU; head shards only, so N > 1) ----
    gather = None
    if world > 1 and (args.gather or args.workload == "long"):
        gather = run_with_gather(args, step, sets, world, stream, B * L)
    # ---- the other workloads, in the same run (default workload only) ----
    subs = None
    if args.workload == "nemotron" and not args.no_sub and not args.shard_of and args.batch is None \
            and args.seqlen is None:
        del pb, sets, step
        torch.cuda.empty_cache()
        subs = sub_results(args, world, rank, dev, stream)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample(w, budget_s=20.0)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": w["name"], "batch": B, "seq_len": L, "n_heads": w["H"],
                       "head_dim": P, "d_state": N, "n_groups": w["G"], "d_conv": K,
                       "chunk_size": Q, "state_dtype": "f32",
                       "shard": f"{H_l} heads / {G_l} groups per GPU",
                       "l2": f"inputs larger than L2: {rot} rotating input/output sets, "
                             f"{step_bytes * rot / 2**20:.0f} MiB touched per rotation"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "peak_source": f"{peak_kind} hbm_gbs",
                         "kernel_ms": kernel_ms, "algorithmic_bytes_per_gpu": alg},
            "gpu_launches": launches,
            "launch": f"CUDA graph replay of one captured step per input set ({per_step} library "
                      f"kernels a step, counted while capturing)",
            "clocks": clocks.summary(h0, h1),
        }
        if e2e is not None:
            line["e2e"] = e2e
        if gather is not None:
            line["with_gather"] = gather
        if subs is not None:
            line["sub_results"] = subs
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_with_gather(args, step, sets, world, stream, tokens):
    """Device-timed steps, each one prefill followed by the all-gather of y
    over the ranks (`sharding.allgather_heads`: one NCCL all-gather into a
    head-major buffer, then a permute to [B, L, H, P]); max over ranks."""
    import torch
    from alloy_b200 import sharding
    rot = len(sets)
    y_bytes = sets[0][1]["y"].numel() * sets[0][1]["y"].element_size()

    def gstep(i):
        step(i)
        sharding.allgather_heads(sets[i % rot][1]["y"], world)

    for i in range(args.warmup):
        gstep(i)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(args.steps):
        gstep(i)
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = dist_max(ev0.elapsed_time(ev1) / args.steps, world)
    return {"value": tokens / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms,
            "collective": "NCCL all_gather of y (head-major) + permute to [B, L, H, P]",
            "bytes_received_per_gpu": y_bytes * (world - 1)}


def nvml_handle(torch_device):
    """The NVML handle of a CUDA device, matched by PCI location (CUDA and NVML
    enumerate devices differently under CUDA_VISIBLE_DEVICES); None without NVML."""
    try:
        import pynvml
        import torch
        pynvml.nvmlInit()
        pr = torch.cuda.get_device_properties(torch_device)
        want = (int(getattr(pr, "pci_domain_id", 0)), int(getattr(pr, "pci_bus_id", -1)),
                int(getattr(pr, "pci_device_id", 0)))
        for i in range(pynvml.nvmlDeviceGetCount()):
            hi = pynvml.nvmlDeviceGetHandleByIndex(i)
            pci = pynvml.nvmlDeviceGetPciInfo(hi)
            if (int(pci.domain), int(pci.bus), int(pci.device)) == want:
                return hi
    except Exception:
        pass
    return None


def gpu_local_cpus(torch_device):
    """The host CPUs on the GPU's side of the machine (NVML's CPU affinity of
    the device), or None when NVML does not say."""
    try:
        import pynvml
        h = nvml_handle(torch_device)
        if h is None:
            return None
        words = (os.cpu_count() + 63) // 64
        mask = pynvml.nvmlDeviceGetCpuAffinity(h, words)
        cpus = {64 * w + b for w, m in enumerate(mask) for b in range(64) if (int(m) >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        return cpus or None
    except Exception:
        return None


def pinned_near(torch_device, shape, dtype):
    """A pinned host tensor whose pages sit on the memory node of the GPU's
    local CPUs: the process is bound to those CPUs while the buffer is
    allocated and first written, then its affinity is restored (DMA from a
    buffer on the other socket crosses the inter-socket link)."""
    import torch
    cpus = gpu_local_cpus(torch_device)
    saved = os.sched_getaffinity(0)
    try:
        if cpus:
            os.sched_setaffinity(0, cpus)
        t = torch.empty(shape, dtype=dtype, pin_memory=True)
        t.zero_()
    finally:
        os.sched_setaffinity(0, saved)
    return t


def run_e2e(args, set0, kw, world, stream, tokens):
    """The same step through the public API with host buffers:
    ``mixer.ssd_combined_streamed`` on pinned host activations, which copies
    each piece of the sequence in, runs the prefill kernels on it and copies
    its y (and, after a row's last piece, the row's states) out, the three
    overlapped on separate streams.  Every byte crosses PCIe inside the
    timed region."""
    import torch
    from alloy_b200 import mixer
    inp, out = set0
    dev = inp["xBC"].device
    host_in = {k: pinned_near(dev, inp[k].shape, inp[k].dtype) for k in ("xBC", "dt_raw")}
    for k in host_in:
        host_in[k].copy_(inp[k])
    host_y = pinned_near(dev, out["y"].shape, out["y"].dtype)
    host_h = pinned_near(dev, out["h"].shape, out["h"].dtype)
    host_cs = pinned_near(dev, out["cs"].shape, out["cs"].dtype)
    local = gpu_local_cpus(dev)
    e2e_steps = max(3, min(args.steps, 10))

    def e2e_step():
        mixer.ssd_combined_streamed(host_in["xBC"], host_in["dt_raw"], inp["conv_w"],
                                    inp["conv_b"], inp["dt_bias"], inp["A_log"], inp["D"],
                                    out=host_y, ssm_state_out=host_h, conv_state_out=host_cs,
                                    piece_tokens=args.piece_tokens, **kw)

    # untimed steps first: they also bring the PCIe link up from its idle speed
    # after the device-only timing above
    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = dist_max(e0.elapsed_time(e1) / e2e_steps, world)
    h2d = sum(t.numel() * t.element_size() for t in host_in.values())
    d2h = sum(t.numel() * t.element_size() for t in (host_y, host_h, host_cs))
    return {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s",
            "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
            "ms_per_step": e2e_ms, "steps": e2e_steps,
            "api": f"mixer.ssd_combined_streamed, pieces of {args.piece_tokens} tokens per row",
            "host_buffers": ("pinned, on the memory node of the GPU's local CPUs "
                             f"({len(local)} of {os.cpu_count()})" if local else
                             "pinned (NVML gave no CPU affinity for the GPU)")}


def run_gated_norm(args, w):
    """Gate + inner RMS norm of the mixer output (y * silu(gate), then the
    full-width RMS norm with a weight): the rows of the workload's tokens split
    over the GPUs; reported as achieved HBM GB/s (y and gate read once, out
    written once).  Inputs rotate through enough sets to exceed 3x L2."""
    import torch
    from alloy_b200 import _lib, mixer

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local if world > 1 else 0)
    D = w["H"] * w["P"]
    rows_total = w["B"] * w["L"]
    if rows_total % world:
        raise SystemExit("rows do not split over the GPUs")
    rows = rows_total // world
    gen = torch.Generator(device=dev)
    gen.manual_seed(11 + rank)
    set_bytes = 3 * rows * D * 2
    rot = max(1, math.ceil(3 * L2_BYTES / set_bytes))
    sets = [(torch.randn((rows, D), generator=gen, device=dev).to(torch.bfloat16),
             torch.randn((rows, D), generator=gen, device=dev).to(torch.bfloat16),
             torch.empty((rows, D), dtype=torch.bfloat16, device=dev)) for _ in range(rot)]
    weight = torch.rand(D, generator=gen, device=dev) + 0.5

    def step(i):
        y, g, o = sets[i % rot]
        mixer.gated_rmsnorm(y, g, weight, eps=1e-5, out=o)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(dev.index)
    clocks.start()
    barrier(world)
    torch.cuda.synchronize()
    h0 = time.perf_counter()
    launches0 = _lib.load().alloy_kernel_launch_count()
    ev0.record(stream)
    for i in range(args.steps):
        step(i)
    ev1.record(stream)
    launches = _lib.load().alloy_kernel_launch_count() - launches0
    torch.cuda.synchronize()
    h1 = time.perf_counter()
    barrier(world)
    clocks.stop()
    ms = dist_max(ev0.elapsed_time(ev1) / args.steps, world)
    alg = 3 * rows * D * 2 + D * 4
    peak, peak_kind = measured_peaks()
    gbs = alg * world / (ms * 1e-3) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": "Mamba-2 gated RMS norm (y * silu(gate), RMSNorm(d_inner)) HBM GB/s",
            "value": gbs, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": w["name"], "rows": rows_total, "channels": D,
                       "norm": "full width, eps 1e-5, fp32 weight",
                       "l2": f"{rot} rotating input/output sets of {set_bytes / 2**20:.0f} MiB"},
            "roofline": {"bound": "hbm", "achieved": gbs / world, "peak": peak, "unit": "GB/s",
                         "frac": gbs / world / peak, "traffic": None,
                         "peak_source": f"{peak_kind} hbm_gbs"},
            "gpu_launches": launches, "clocks": clocks.summary(h0, h1)}), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_proj(args, w):
    """The layer's two projections over all tokens of the prefill step:
    in_proj [B*L, d_model] x [d_model, 2*d_inner + 2*G*N + H] and out_proj
    [B*L, d_inner] x [d_inner, d_model] (``mixer.linear``, the tcgen05 GEMM);
    tokens split over the GPUs.  Reported as TFLOP/s of the two products; the
    same step through torch (cuBLAS) is timed beside it in the same run."""
    import torch
    from alloy_b200 import _lib, mixer

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local if world > 1 else 0)
    d_model, d_inner = w["d_model"], w["H"] * w["P"]
    n_in = 2 * d_inner + 2 * w["G"] * w["N"] + w["H"]
    rows_total = w["B"] * w["L"]
    if rows_total % world:
        raise SystemExit("rows do not split over the GPUs")
    M = rows_total // world
    gen = torch.Generator(device=dev)
    gen.manual_seed(13 + rank)

    def rnd(*shape, scale=1.0):
        return (torch.randn(shape, generator=gen, device=dev) * scale).to(torch.bfloat16)

    x_in, w_in = rnd(M, d_model), rnd(n_in, d_model, scale=d_model ** -0.5)
    x_out, w_out = rnd(M, d_inner), rnd(d_model, d_inner, scale=d_inner ** -0.5)
    y_in = torch.empty((M, n_in), dtype=torch.bfloat16, device=dev)
    y_out = torch.empty((M, d_model), dtype=torch.bfloat16, device=dev)
    flops = 2.0 * M * (d_model * n_in + d_inner * d_model)

    def ours(i):
        mixer.linear(x_in, w_in, out=y_in)
        mixer.linear(x_out, w_out, out=y_out)

    def cublas(i):
        torch.matmul(x_in, w_in.t(), out=y_in)
        torch.matmul(x_out, w_out.t(), out=y_out)

    stream = torch.cuda.current_stream(dev)

    def timed(step, clocks=None):
        for i in range(args.warmup):
            step(i)
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if clocks:
            clocks.start()
        barrier(world)
        torch.cuda.synchronize()
        h0 = time.perf_counter()
        n0 = _lib.load().alloy_kernel_launch_count()
        ev0.record(stream)
        for i in range(args.steps):
            step(i)
        ev1.record(stream)
        n = _lib.load().alloy_kernel_launch_count() - n0
        torch.cuda.synchronize()
        h1 = time.perf_counter()
        barrier(world)
        if clocks:
            clocks.stop()
        return dist_max(ev0.elapsed_time(ev1) / args.steps, world), n, (h0, h1)

    # the reported number first; then cuBLAS and the library again in both
    # orders, so that neither side gets the cooler GPU (a 1 kW part runs these
    # products at its power cap)
    clocks = ClockSampler(dev.index)
    ms, launches, (h0, h1) = timed(ours, clocks)
    ref_a, _, _ = timed(cublas)
    ref_b, _, _ = timed(cublas)
    ms_b, _, _ = timed(ours)
    ref_ms = (ref_a + ref_b) / 2
    ours_pair_ms = (ms + ms_b) / 2
    # parity on a slice of rows against the fp32 product
    rows = slice(0, 512)
    ref = x_in[rows].float() @ w_in.float().t()
    rel = ((y_in[rows].float() - ref).norm() / ref.norm()).item()
    tflops = flops * world / (ms * 1e-3) / 1e12
    peak, peak_kind = measured_tensor_peak(sustained=True)
    if rank == 0:
        print(json.dumps({
            "metric": "Mamba-2 layer in_proj + out_proj (prefill) TFLOP/s",
            "value": tflops, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": w["name"], "tokens": rows_total, "d_model": d_model,
                       "in_features_out": n_in, "d_inner": d_inner,
                       "l2": "operands 1.3 GB a step, larger than L2"},
            "cublas_ms_per_step": ref_ms, "ours_ms_per_step_interleaved": ours_pair_ms,
            "speedup_vs_cublas": ref_ms / ours_pair_ms,
            "comparison": "library, cuBLAS, cuBLAS, library: K steps each, means of the two of each",
            "rel_l2_vs_fp32": rel,
            "roofline": {"bound": "tensor", "achieved": tflops / world, "peak": peak,
                         "unit": "TFLOP/s", "frac": tflops / world / peak, "traffic": None,
                         "peak_source": peak_kind},
            "gpu_launches": launches, "clocks": clocks.summary(h0, h1)}), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_conv(args, w):
    """The standalone causal depthwise conv1d + SiLU (``mixer.conv1d_silu``, the
    split-mode kernel of the reference's ``fused_conv1d_silu``) over the layer's
    xBC (conv_dim = H P + 2 G N channels).  Batch rows split over the GPUs;
    reported as achieved HBM GB/s (x_padded read once, out written once).
    Inputs rotate through enough sets to exceed 3x L2."""
    import torch
    from alloy_b200 import _lib, mixer

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local if world > 1 else 0)
    B, L, K = w["B"], w["L"], w["K"]
    C = w["H"] * w["P"] + 2 * w["G"] * w["N"]
    if B % world:
        raise SystemExit("batch rows do not split over the GPUs")
    Bl = B // world
    gen = torch.Generator(device=dev)
    gen.manual_seed(31 + rank)
    set_bytes = Bl * (2 * L + K - 1) * C * 2
    rot = max(1, math.ceil(3 * L2_BYTES / set_bytes))
    sets = [(torch.randn((Bl, L + K - 1, C), generator=gen, device=dev).to(torch.bfloat16),
             torch.empty((Bl, L, C), dtype=torch.bfloat16, device=dev)) for _ in range(rot)]
    weight = torch.randn((C, K), generator=gen, device=dev) * 0.5
    bias = torch.zeros(C, device=dev)

    def step(i):
        x, out = sets[i % rot]
        mixer.conv1d_silu(x, weight, bias, L, out=out)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(dev.index)
    clocks.start()
    barrier(world)
    torch.cuda.synchronize()
    h0 = time.perf_counter()
    launches0 = _lib.load().alloy_kernel_launch_count()
    ev0.record(stream)
    for i in range(args.steps):
        step(i)
    ev1.record(stream)
    launches = _lib.load().alloy_kernel_launch_count() - launches0
    torch.cuda.synchronize()
    h1 = time.perf_counter()
    barrier(world)
    clocks.stop()
    ms = dist_max(ev0.elapsed_time(ev1) / args.steps, world)
    alg = set_bytes + C * (K + 1) * 4
    peak, peak_kind = measured_peaks()
    gbs = alg * world / (ms * 1e-3) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": "Mamba-2 causal depthwise conv1d+SiLU HBM GB/s",
            "value": gbs, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": w["name"], "batch": B, "seq_len": L, "channels": C, "d_conv": K,
                       "l2": f"{rot} rotating input/output sets of {set_bytes / 2**20:.0f} MiB"},
            "roofline": {"bound": "hbm", "achieved": gbs / world, "peak": peak, "unit": "GB/s",
                         "frac": gbs / world / peak, "traffic": None,
                         "peak_source": f"{peak_kind} hbm_gbs"},
            "gpu_launches": launches, "clocks": clocks.summary(h0, h1)}), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_scan_bwd(args, w):
    """Backward of the selective scan (``mixer.selective_scan_backward``: the
    forward recomputed, two time-reversed scans and one forward scan on the fp32
    CUDA-core scan kernel, the log-decay gradient as a reverse cumulative sum)
    on fp32 inputs of the workload's shape; tokens/s of the backward.  Batch
    rows split over the GPUs."""
    import torch
    from alloy_b200 import _lib, mixer

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local if world > 1 else 0)
    B, L, H, P, N, G = w["B"], w["L"], w["H"], w["P"], w["N"], w["G"]
    if B % world:
        raise SystemExit("batch rows do not split over the GPUs")
    Bl = B // world
    gen = torch.Generator(device=dev)
    gen.manual_seed(41 + rank)
    bf16 = w.get("dtype") == "bf16"
    act = torch.bfloat16 if bf16 else torch.float32
    x = (torch.randn((Bl, L, H, P), generator=gen, device=dev) * 0.5).to(act)
    Bm = torch.randn((Bl, L, G, N), generator=gen, device=dev).to(act)
    Cm = torch.randn((Bl, L, G, N), generator=gen, device=dev).to(act)
    la = -torch.rand((Bl, L, H), generator=gen, device=dev) * 0.1
    dy = torch.randn((Bl, L, H, P), generator=gen, device=dev).to(act)

    def step(i):
        mixer.selective_scan_backward(x, None, Bm, Cm, dy, log_a=la)

    # the variant with the log-decay gradient's scans on the fp32 scan
    fast_ms = None
    if bf16:
        for i in range(2):
            mixer.selective_scan_backward(x, None, Bm, Cm, dy, log_a=la, tensor_core_log_decay=False)
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        f0.record()
        for i in range(5):
            mixer.selective_scan_backward(x, None, Bm, Cm, dy, log_a=la, tensor_core_log_decay=False)
        f1.record()
        torch.cuda.synchronize()
        fast_ms = f0.elapsed_time(f1) / 5

    # one forward scan alone (the unit the backward runs four times), for its roofline:
    # algorithmic bytes = x, B, C, log decay read once, y (fp32) written once
    def one_scan():
        mixer.selective_scan(x, None, Bm, Cm, log_a=la, out_dtype=torch.float32, write_ssm_state=False)

    for i in range(3):
        one_scan()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for i in range(max(args.steps, 5)):
        one_scan()
    e1.record()
    torch.cuda.synchronize()
    scan_ms = e0.elapsed_time(e1) / max(args.steps, 5)
    scan_bytes = Bl * L * (H * P * x.element_size() + 2 * G * N * Bm.element_size() + 4 * H + 4 * H * P)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(dev.index)
    clocks.start()
    barrier(world)
    torch.cuda.synchronize()
    h0 = time.perf_counter()
    launches0 = _lib.load().alloy_kernel_launch_count()
    ev0.record(stream)
    for i in range(args.steps):
        step(i)
    ev1.record(stream)
    launches = _lib.load().alloy_kernel_launch_count() - launches0
    torch.cuda.synchronize()
    h1 = time.perf_counter()
    barrier(world)
    clocks.stop()
    ms = dist_max(ev0.elapsed_time(ev1) / args.steps, world)
    tokens = B * L
    if rank == 0:
        peak, src = measured_peaks()
        achieved = scan_bytes / (scan_ms * 1e-3) / 1e9
        print(json.dumps({
            "metric": "Mamba-2 selective scan backward tokens/s (%s)" % ("bf16" if bf16 else "fp32"),
            "value": tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16" if bf16 else "f32",
            "data": "synthetic",
            "config": {"workload": w["name"], "batch": B, "seq_len": L, "n_heads": H,
                       "head_dim": P, "d_state": N, "n_groups": G,
                       "path": ("4 tcgen05 scans (bf16 operands; the recomputed forward and dx, which "
                                "feed the log-decay gradient, with bf16-pair operands)" if bf16 else
                                "4 fp32 CUDA-core scans") + " + reverse cumulative sum"},
            "fp32_log_decay_ms": fast_ms,
            "one_scan": {"ms": scan_ms, "bytes": scan_bytes,
                         "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                                      "frac": achieved / peak, "peak_source": src}},
            "gpu_launches": launches, "clocks": clocks.summary(h0, h1)}), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_conv_bwd(args, w):
    """Backward of conv1d + SiLU over the layer's xBC (conv_dim = H P + 2 G N
    channels): dx_padded, dweight, dbias from dy.  Batch rows split over the
    GPUs; reported as achieved HBM GB/s (x_padded and dy read once, dx_padded
    written once).  Inputs rotate through enough sets to exceed 3x L2."""
    import torch
    from alloy_b200 import _lib, mixer

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local if world > 1 else 0)
    B, L, K = w["B"], w["L"], w["K"]
    C = w["H"] * w["P"] + 2 * w["G"] * w["N"]
    if B % world:
        raise SystemExit("batch rows do not split over the GPUs")
    Bl = B // world
    gen = torch.Generator(device=dev)
    gen.manual_seed(21 + rank)
    set_bytes = Bl * (2 * (L + K - 1) + L) * C * 2
    rot = max(1, math.ceil(3 * L2_BYTES / set_bytes))
    sets = [(torch.randn((Bl, L + K - 1, C), generator=gen, device=dev).to(torch.bfloat16),
             torch.randn((Bl, L, C), generator=gen, device=dev).to(torch.bfloat16),
             torch.empty((Bl, L + K - 1, C), dtype=torch.bfloat16, device=dev)) for _ in range(rot)]
    weight = torch.randn((C, K), generator=gen, device=dev) * 0.5
    bias = torch.zeros(C, device=dev)

    def step(i):
        x, dy, dx = sets[i % rot]
        mixer.conv1d_silu_backward(x, weight, bias, dy, dx_out=dx)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(dev.index)
    clocks.start()
    barrier(world)
    torch.cuda.synchronize()
    h0 = time.perf_counter()
    launches0 = _lib.load().alloy_kernel_launch_count()
    ev0.record(stream)
    for i in range(args.steps):
        step(i)
    ev1.record(stream)
    launches = _lib.load().alloy_kernel_launch_count() - launches0
    torch.cuda.synchronize()
    h1 = time.perf_counter()
    barrier(world)
    clocks.stop()
    ms = dist_max(ev0.elapsed_time(ev1) / args.steps, world)
    alg = set_bytes + 2 * C * (K + 1) * 4
    peak, peak_kind = measured_peaks()
    gbs = alg * world / (ms * 1e-3) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": "Mamba-2 conv1d+SiLU backward (dx, dweight, dbias) HBM GB/s",
            "value": gbs, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": w["name"], "batch": B, "seq_len": L, "channels": C, "d_conv": K,
                       "l2": f"{rot} rotating input/output sets of {set_bytes / 2**20:.0f} MiB"},
            "roofline": {"bound": "hbm", "achieved": gbs / world, "peak": peak, "unit": "GB/s",
                         "frac": gbs / world / peak, "traffic": None,
                         "peak_source": f"{peak_kind} hbm_gbs"},
            "gpu_launches": launches, "clocks": clocks.summary(h0, h1)}), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_decode_block(args, w):
    """One Nemotron-H Mamba layer (d_model 4096, in-projection, cached step,
    gate + inner norm, out-projection; random bf16 weights) decoding B
    sequences after an L-token prefill: tokens/s with the step replayed from a
    CUDA graph (`MambaDecodeGraph`), and eagerly.  Batch 1 is weight-bound: the
    projections' 219 MB of weights are read once per token."""
    import torch
    from alloy_b200 import _lib
    from alloy_b200.decode_graph import MambaDecodeGraph
    from alloy_b200.mamba_block import MambaBlock, MambaCache

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local if world > 1 else 0)
    H, P, N, G, K = w["H"], w["P"], w["N"], w["G"], w["K"]
    B = w["B"]
    torch.manual_seed(5 + rank)
    blk = MambaBlock(d_model=H * P // 2, d_state=N, d_conv=K, expand=2, headdim=P, n_groups=G,
                     use_D=True, use_inner_norm=True, combined_proj=True, device=dev,
                     dtype=torch.bfloat16)
    with torch.no_grad():
        blk.A_log.uniform_(0.0, math.log(16.0))
        blk.dt_bias.uniform_(-6.0, -2.0)
        blk.D.normal_()
        blk.conv_weight.normal_(0, 0.5)
    T = 64
    xs = torch.randn((T, B, 1, blk.d_model), device=dev, dtype=torch.bfloat16)
    cache = MambaCache()
    with torch.no_grad():
        blk(torch.randn((B, w["L"], blk.d_model), device=dev, dtype=torch.bfloat16), cache=cache)
    graph = MambaDecodeGraph(blk, cache, batch=B)
    stream = torch.cuda.current_stream(dev)

    def timed(fn):
        for i in range(args.warmup):
            fn(i)
        torch.cuda.synchronize()
        barrier(world)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n0 = _lib.load().alloy_kernel_launch_count()
        ev0.record(stream)
        for i in range(args.steps):
            fn(i)
        ev1.record(stream)
        n = _lib.load().alloy_kernel_launch_count() - n0
        torch.cuda.synchronize()
        barrier(world)
        return dist_max(ev0.elapsed_time(ev1) / args.steps, world), n

    with torch.no_grad():
        ms_eager, n_eager = timed(lambda i: blk(xs[i % T], cache=cache))
        clocks = ClockSampler(dev.index)
        clocks.start()
        h0 = time.perf_counter()
        ms_graph, _ = timed(lambda i: graph.step(xs[i % T]))
        h1 = time.perf_counter()
        clocks.stop()
    weights = sum(p.numel() * p.element_size() for p in (blk.in_proj.weight, blk.out_proj.weight))
    alg = weights + 2 * cache.ssm_state.numel() * 4 + 2 * cache.conv_state.numel() * 2
    peak, peak_kind = measured_peaks()
    gbs = alg / (ms_graph * 1e-3) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": "Mamba-2 layer decode tokens/s (Nemotron-H layer, batch 1, CUDA graph)",
            "value": B * world / (ms_graph * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_graph,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random weights)",
            "config": {"workload": w["name"], "batch": B, "prefill": w["L"], "d_model": blk.d_model,
                       "n_heads": H, "head_dim": P, "d_state": N, "n_groups": G,
                       "weights_mb": round(weights / 1e6, 1)},
            "eager": {"value": B * world / (ms_eager * 1e-3), "unit": "tokens/s",
                      "ms_per_step": ms_eager, "alloy_launches_per_step": n_eager / args.steps},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                         "frac": gbs / peak, "traffic": None, "peak_source": f"{peak_kind} hbm_gbs",
                         "note": "bytes per step = projection weights + state and conv cache read and written"},
            "gpu_launches": "graph replays: " + str(args.steps),
            "clocks": clocks.summary(h0, h1)}), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def decode_problem(w, world, rank, dev):
    """This rank's share of the decode workload (batch rows split over the
    ranks): B sequences advance one token per step through the conv cache and
    the fp32 SSM cache ([B, H, P, N] storage), 64 tokens cycled."""
    import torch
    from alloy_b200 import mixer
    H, P, N, G, K = w["H"], w["P"], w["N"], w["G"], w["K"]
    if w["B"] % world:
        raise SystemExit("batch does not split over the GPUs")
    B = w["B"] // world
    C = H * P + 2 * G * N
    gen = torch.Generator(device=dev)
    gen.manual_seed(7 + rank)
    state_pn = torch.randn((B, H, P, N), generator=gen, device=dev) * math.sqrt(0.1)
    conv_ck = torch.randn((B, C, K - 1), generator=gen, device=dev).to(torch.bfloat16)
    T = 64
    xtok = torch.randn((T, B, C), generator=gen, device=dev).to(torch.bfloat16)
    dtok = torch.randn((T, B, H), generator=gen, device=dev).to(torch.bfloat16)
    p = make_prefill_inputs(1, 1, H, P, N, G, K, seed=3, device=dev)
    y = torch.empty((B, H, P), dtype=torch.bfloat16, device=dev)
    ssm, conv = state_pn.transpose(2, 3), conv_ck.transpose(1, 2)
    kw = dict(n_heads=H, head_dim=P, d_state=N, n_groups=G, out=y)

    def step(i):
        mixer.ssd_decode_step(xtok[i % T], dtok[i % T], p["conv_w"], p["conv_b"], p["dt_bias"],
                              p["A_log"], p["D"], conv, ssm, **kw)

    # state read + written, conv cache read + written, the token in, y out
    alg = (2 * B * H * P * N * 4 + 2 * B * C * (K - 1) * 2 + B * C * 2 + B * H * 2
           + B * H * P * 2)
    return dict(B=B, C=C, T=T, step=step, alg=alg,
                state_mib=B * H * P * N * 4 / 2**20)


def run_decode(args, w):
    """Decode-step workload: B sequences advance one token per step through
    the conv cache and the fp32 SSM cache ([B, H, P, N] storage), 64
    sequential tokens cycled; reported as achieved HBM GB/s (the state is
    read and written once per token)."""
    import torch

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local if world > 1 else 0)
    H, P, N, G, K = w["H"], w["P"], w["N"], w["G"], w["K"]
    dp = decode_problem(w, world, rank, dev)
    stream = torch.cuda.current_stream(dev)
    for i in range(args.warmup):
        dp["step"](i)
    torch.cuda.synchronize()
    clocks = ClockSampler(dev.index)
    clocks.start()
    h0 = time.perf_counter()
    ms, _, launches = time_steps(dp["step"], args.steps, 0, world, stream, per_step_events=False)
    h1 = time.perf_counter()
    clocks.stop()
    ms = dist_max(ms, world)
    alg = dp["alg"]
    peak, peak_kind = measured_peaks()
    gbs = alg * world / (ms * 1e-3) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": "Mamba-2 decode step (state update + conv-cache roll) HBM GB/s",
            "value": gbs, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": w["name"], "batch": w["B"], "n_heads": H, "head_dim": P,
                       "d_state": N, "n_groups": G, "state_layout": "[B,H,P,N] f32",
                       "conv_state_layout": "[B,C,K-1] bf16", "tokens_cycled": dp["T"],
                       "l2": "state of %.0f MiB per GPU > L2" % dp["state_mib"]},
            "roofline": {"bound": "hbm", "achieved": gbs / world, "peak": peak, "unit": "GB/s",
                         "frac": gbs / world / peak, "traffic": None,
                         "peak_source": f"{peak_kind} hbm_gbs"},
            "gpu_launches": launches, "clocks": clocks.summary(h0, h1)}), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# ------------------------------------------------------------------ CPU reference
def _all_blas_threads():
    """Every host core for the numpy BLAS of the CPU samples (torchrun sets
    OMP_NUM_THREADS=1 for its ranks; the reference arm runs on rank 0 alone)."""
    import contextlib
    try:
        from threadpoolctl import threadpool_limits
        return threadpool_limits(limits=os.cpu_count() or 1, user_api="blas")
    except Exception:
        return contextlib.nullcontext()


def _blas_threads():
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        return max(n) if n else 1
    except Exception:
        return os.cpu_count() or 1


def _cpu_sample(w, heads, tokens, seed=0):
    """Time the reference algorithm (oracle.mixer_core: conv -> discretise ->
    chunked state-space scan -> D) on one batch row, ``heads`` heads of one
    group, ``tokens`` tokens.  Returns seconds."""
    import oracle
    inp = oracle.make_inputs(B=1, L=tokens, H=heads, P=w["P"], N=w["N"], G=1, dtype="bf16",
                             seed=seed)
    t0 = time.perf_counter()
    oracle.mixer_core(inp["xBC"], inp["dt_raw"], inp["conv_weight"], inp["conv_bias"],
                      inp["dt_bias"], inp["A_log"], inp["D"], n_heads=heads, headdim=w["P"],
                      d_state=w["N"], n_groups=1, chunk_size=w["Q"])
    return time.perf_counter() - t0


def cpu_baseline_sample(w, budget_s=20.0):
    with _all_blas_threads():
        return _cpu_baseline_sample(w, budget_s)


def _cpu_baseline_sample(w, budget_s):
    heads = w["H"] // w["G"]           # one head-group
    tokens = min(w["L"], 2 * w["Q"])   # the first chunks of one batch row
    secs = _cpu_sample(w, heads, tokens)
    reps = 1
    while secs * (reps + 1) < budget_s and reps < 4:
        secs = min(secs, _cpu_sample(w, heads, tokens, seed=reps))
        reps += 1
    per_layer_tokens_s = tokens / (secs * w["H"] / heads)
    return {"value": per_layer_tokens_s, "unit": "tokens/s", "cores": _blas_threads(),
            "kind": "port",
            "sample": f"oracle.mixer_core (the reference's chunked state-space scan, numpy fp32) "
                      f"on 1 batch row x {heads} heads (one group) x {tokens} tokens, "
                      f"best of {reps}; extrapolated linearly to all {w['H']} heads"}


def run_reference(args, w):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    with _all_blas_threads():
        _run_reference(args, w, world)


def _run_reference(args, w, world):
    heads = w["H"] // w["G"]
    tokens = min(w["L"], w["Q"])
    # size each step so that warmup + steps stay within about two minutes
    probe = _cpu_sample(w, 1, tokens)
    per_head = max(probe, 1e-3)
    budget_per_step = 120.0 / max(1, args.steps + args.warmup)
    heads = max(1, min(heads, int(budget_per_step / per_head)))
    for i in range(args.warmup):
        _cpu_sample(w, heads, tokens, seed=i)
    total = 0.0
    for i in range(args.steps):
        total += _cpu_sample(w, heads, tokens, seed=100 + i)
    secs = total / args.steps
    value = tokens / (secs * w["H"] / heads)
    cores = _blas_threads()
    sample = (f"oracle.mixer_core (numpy restatement of alloy's mamba_block.py conv + "
              f"discretise + chunked state-space scan + D; MLX is not installable here) on "
              f"1 batch row x {heads} heads x {tokens} tokens per step, extrapolated "
              f"linearly to {w['H']} heads")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": secs * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": w["name"], "batch": w["B"], "seq_len": w["L"],
                       "n_heads": w["H"], "head_dim": w["P"], "d_state": w["N"],
                       "n_groups": w["G"], "chunk_size": w["Q"]},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "gpu_launches": 0}
    print(json.dumps(line), flush=True)


def main():
    faulthandler.enable()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="nemotron")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg")
    ap.add_argument("--shard-of", type=int, default=None,
                    help="on one GPU, run the share of one rank of an N-GPU prefill (for profiling "
                         "the per-GPU work of a multi-GPU run; the line reports that shard's tokens)")
    ap.add_argument("--piece-tokens", type=int, default=2048,
                    help="tokens per piece of the end-to-end leg's host-streamed prefill")
    ap.add_argument("--no-sub", action="store_true",
                    help="skip the other workloads' sub-results of the default run")
    ap.add_argument("--gather", action="store_true",
                    help="also time each step followed by the all-gather of y (N > 1; "
                         "always on for the long workload)")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the workload's batch (smaller cases for profiling)")
    ap.add_argument("--seqlen", type=int, default=None,
                    help="override the workload's sequence length")
    args = ap.parse_args()
    if args.impl == "reference":
        # the CPU arm uses every host core: torchrun sets OMP_NUM_THREADS=1 for
        # its ranks, and numpy's BLAS sizes its thread pool when it loads
        for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
            os.environ[var] = str(os.cpu_count() or 1)
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    w = dict(WORKLOADS[args.workload])
    if args.batch is not None:
        w["B"] = args.batch
    if args.seqlen is not None:
        w["L"] = args.seqlen
    if args.shard_of:
        w["name"] += f"_shard_of_{args.shard_of}"
    if args.batch is not None or args.seqlen is not None:
        w["name"] += f"_b{w['B']}_l{w['L']}"
    if args.impl == "reference":
        run_reference(args, w)
    elif args.workload == "decode":
        run_decode(args, w)
    elif args.workload == "gated_norm":
        run_gated_norm(args, w)
    elif args.workload == "decode_block":
        run_decode_block(args, w)
    elif args.workload == "conv_bwd":
        run_conv_bwd(args, w)
    elif args.workload == "conv":
        run_conv(args, w)
    elif args.workload == "proj":
        run_proj(args, w)
    elif args.workload in ("scan_bwd", "scan_bwd_bf16"):
        run_scan_bwd(args, w)
    else:
        run_ours(args, w)


if __name__ == "__main__":
    main()
