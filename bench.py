#!/usr/bin/env python
"""Causal self-attention forward + backward throughput on B200.

Workload (per GPU, weak scaling): the attention of kerr-engine's 768-dim model,
n_embd 768 = 12 heads x head_dim 64, seq_len 256, batch 16 sequences, 4 blocks.
One step = the 4 blocks' attention forwards followed by their backwards in
reverse order, exactly the attention work of one training step
(src/pipeline.rs:177-758).  Each block has its own q|k|v, o, lse, dout and
dq|dk|dv buffers (~101 MB per block, ~404 MB per step > the 126 MB L2), so no
L2 flush is needed between steps.  Inputs are seeded synthetic q, k, v ~
N(0,1)/8 and dout ~ N(0,1) (no checkpoint or corpus is available).

metric: tokens/s = (sequences x seq_len x ranks) / step time (CUDA events,
max over ranks).  e2e: the same through the host-buffer C ABI calls
(kattn_fwd_host_save / kattn_bwd_host_saved, the forward state kept on the
device as the reference's AttnCache; e2e_plain: kattn_fwd_host /
kattn_bwd_host), host<->device copies inside the timed region.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "kerr-engine_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "causal-attn fwd+bwd tokens/s per GPU at 768-dim T=256; % of roofline; 1/2/4/8 GPU"
WORKLOAD = {"workload": "kerr-engine 768-dim attention fwd+bwd, 4 blocks per step",
            "batch_per_gpu": 16, "seq_len": 256, "n_head": 12, "head_dim": 64, "n_embd": 768, "blocks": 4,
            "causal": True, "layout": "q|k|v column blocks of one [B*T][3C] buffer (ld 3C)",
            "l2": "no flush: 4 blocks x ~101 MB of distinct buffers per step exceed the 126 MB L2"}
FALLBACK_HBM_GBS = 6650.0


def algorithmic(B, T, H, d):
    """Per-block algorithmic work (causal, no recompute counted):
    flops: 2 GEMM-like products forward (QK^T, PV) and 4 backward (dV, dP, dQ, dK),
    each 2*d per (query, key<=query) pair; bytes: forward reads q,k,v and writes
    o, lse; backward reads q,k,v,o,dout,lse and writes dq,dk,dv."""
    pairs = T * (T + 1) / 2
    slabs = B * H
    return {
        "fwd_flops": 2 * 2 * d * pairs * slabs,
        "bwd_flops": 4 * 2 * d * pairs * slabs,
        "fwd_bytes": 4 * (4 * T * d + T) * slabs,
        "bwd_bytes": 4 * (8 * T * d + T) * slabs,
    }


class ClockSampler(threading.Thread):
    """Samples SM clock and clock-event reasons through NVML while running."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.01):
        super().__init__(daemon=True)
        self.period = period_s
        self.samples = []
        self.reasons = set()
        self._halt = threading.Event()
        self.max_mhz = None
        self.ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # NVML missing: clocks reported as unavailable
            self.err = str(e)

    def sample(self):
        nv = self._nv
        self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
        mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
        for bit, name in self.REASONS.items():
            if mask & bit:
                self.reasons.add(name)

    def run(self):
        if not self.ok:
            return
        while not self._halt.is_set():
            try:
                self.sample()
            except Exception:
                pass
            time.sleep(self.period)

    def stop(self):
        self._halt.set()
        if self.ok:
            self.join(timeout=2)
            if not self.samples:
                self.sample()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": "NVML unavailable"}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons - {"gpu_idle"}),
                "samples": len(self.samples)}


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": FALLBACK_HBM_GBS}, "fallback"


def profiled_traffic(*names: str):
    """Sum of the DRAM bytes per launch (read + write) that the committed ncu
    summary profiles/traffic.txt records for the named kernels; None if any
    is missing.  Lines read: `<kernel> <bytes per launch> ...`."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    if not os.path.exists(path):
        return None
    table = {}
    with open(path) as f:
        for line in f:
            parts = line.split()
            if len(parts) >= 2 and not line.startswith("#"):
                try:
                    table[parts[0]] = float(parts[1])
                except ValueError:
                    pass
    if not all(n in table for n in names):
        return None
    return sum(table[n] for n in names)


def cpu_sample(n_seq: int, T: int, H: int, d: int, seed: int = 7):
    """One block's attention fwd+bwd through the oracle over n_seq sequences on
    n_seq host threads (one thread per sequence, as src/train.rs:241-255)."""
    import numpy as np

    from oracle import oracle

    C = H * d
    rng = np.random.default_rng(seed)
    qkv = (rng.standard_normal((n_seq, T, 3 * C)) / 8).astype(np.float32)
    dout = rng.standard_normal((n_seq, T, C)).astype(np.float32)
    q, k, v = qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]
    t0 = time.perf_counter()
    o, att, _ = oracle.forward(q, k, v, H, threads=n_seq)
    oracle.backward(dout, q, k, v, att, H, threads=n_seq)
    return time.perf_counter() - t0


def run_reference(args):
    """The reference's CPU path (oracle port) on this host's cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    W = WORKLOAD
    cores = os.cpu_count() or 1
    n_seq = min(cores, W["batch_per_gpu"])
    from oracle import oracle

    oracle.build()
    for _ in range(args.warmup):
        cpu_sample(n_seq, W["seq_len"], W["n_head"], W["head_dim"])
    times = [cpu_sample(n_seq, W["seq_len"], W["n_head"], W["head_dim"]) for _ in range(args.steps)]
    t = sum(times) / len(times)
    tok_s = n_seq * W["seq_len"] / (W["blocks"] * t)
    step_ms = 1e3 * t * W["blocks"] * math.ceil(W["batch_per_gpu"] / n_seq)
    sample = (f"each step: 1 of 4 blocks, {n_seq} of {W['batch_per_gpu']} sequences in parallel "
              f"(one host thread each); tokens/s scaled to the 4-block step")
    line = {"metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": W, "impl": "reference",
            "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": n_seq, "kind": "port",
                             "sample": sample},
            "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    import kerr_attn
    from kerr_attn.dist import max_over_ranks as _max_over_ranks
    from kerr_attn.dist import sync as _sync
    from kerr_attn.dist import world as _world

    rank, local, world = _world()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 under torchrun")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)

    W = WORKLOAD
    B, T, H, d, NB = W["batch_per_gpu"], W["seq_len"], W["n_head"], W["head_dim"], W["blocks"]
    C = H * d
    ctx = kerr_attn.Context(local)
    ctx.set_path({"auto": kerr_attn.PATH_AUTO, "ffma": kerr_attn.PATH_FFMA,
                  "tensor": kerr_attn.PATH_TENSOR}[args.path])

    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    blocks = []
    for _ in range(NB):
        qkv = torch.randn(B, T, 3 * C, device=dev, generator=g) / 8
        blocks.append({
            "qkv": qkv, "o": torch.empty(B, T, C, device=dev), "lse": torch.empty(B, H, T, device=dev),
            "dout": torch.randn(B, T, C, device=dev, generator=g), "dqkv": torch.empty_like(qkv)})
    for blk in blocks:
        blk["q"], blk["k"], blk["v"] = kerr_attn.split_qkv(blk["qkv"], C)
        blk["dq"], blk["dk"], blk["dv"] = kerr_attn.split_qkv(blk["dqkv"], C)
    stream = torch.cuda.current_stream(dev)

    def step(ev=None):
        n = 0
        for i, blk in enumerate(blocks):
            if ev is not None:
                ev["f"][i][0].record(stream)
            n += kerr_attn.fwd(ctx, blk["q"], blk["k"], blk["v"], blk["o"], blk["lse"], H, stream=stream)
            if ev is not None:
                ev["f"][i][1].record(stream)
        for i in reversed(range(NB)):
            blk = blocks[i]
            if ev is not None:
                ev["b"][i][0].record(stream)
            n += kerr_attn.bwd(ctx, blk["q"], blk["k"], blk["v"], blk["o"], blk["dout"], blk["lse"],
                               blk["dq"], blk["dk"], blk["dv"], H, stream=stream)
            if ev is not None:
                ev["b"][i][1].record(stream)
        return n

    def sync_all():
        _sync(dev)

    def max_over_ranks(x: float) -> float:
        return _max_over_ranks(x, dev)

    for _ in range(args.warmup):
        step()
    sync_all()

    mk = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    # Headline: K steps back to back, nothing recorded between the launches
    # (an event between two kernels would cut the programmatic-launch overlap).
    clocks = ClockSampler(local)
    clocks.start()
    t_start, t_end = mk(), mk()
    sync_all()
    t_start.record(stream)
    launches = 0
    for _ in range(args.steps):
        launches += step()
    t_end.record(stream)
    torch.cuda.synchronize(dev)
    clocks.stop()
    sync_all()
    ms_total = max_over_ranks(t_start.elapsed_time(t_end))
    ms_step = ms_total / args.steps
    # Per-call breakdown for the roofline: the same K steps again with an
    # event pair around every kattn_fwd / kattn_bwd call (launch gaps included).
    evs = [{"f": [(mk(), mk()) for _ in range(NB)], "b": [(mk(), mk()) for _ in range(NB)]}
           for _ in range(args.steps)]
    sync_all()
    e_start, e_end = mk(), mk()
    e_start.record(stream)
    for s in range(args.steps):
        step(evs[s])
    e_end.record(stream)
    torch.cuda.synchronize(dev)
    sync_all()
    ms_step_ev = max_over_ranks(e_start.elapsed_time(e_end)) / args.steps
    fwd_ms = statistics.mean(e["f"][i][0].elapsed_time(e["f"][i][1]) for e in evs for i in range(NB))
    bwd_ms = statistics.mean(e["b"][i][0].elapsed_time(e["b"][i][1]) for e in evs for i in range(NB))
    fwd_ms, bwd_ms = max_over_ranks(fwd_ms), max_over_ranks(bwd_ms)
    tokens_per_step = B * T * world
    value = tokens_per_step / (ms_step / 1e3)

    # End to end through the host-buffer ABI (pinned host inputs and outputs).
    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    hb = []
    for blk in blocks:
        h = {k: blk[k].cpu().pin_memory() for k in ("qkv", "dout")}
        h["o"] = torch.empty(B, T, C).pin_memory()
        h["lse"] = torch.empty(B, H, T).pin_memory()
        h["dqkv"] = torch.empty(B, T, 3 * C).pin_memory()
        h["q"], h["k"], h["v"] = kerr_attn.split_qkv(h["qkv"], C)
        h["dq"], h["dk"], h["dv"] = kerr_attn.split_qkv(h["dqkv"], C)
        hb.append(h)

    # The saved-state pair (the reference's AttnCache flow): each block's
    # forward keeps q/k/v, o and lse on the device for its backward, which
    # then sends only dout up.  The plain pair re-sends everything.
    saved = [kerr_attn.Saved(ctx) for _ in hb]

    def step_host():
        for h, sv in zip(hb, saved):
            kerr_attn.fwd_host_save(ctx, sv, h["q"], h["k"], h["v"], h["o"], h["lse"], H)
        for h, sv in zip(reversed(hb), reversed(saved)):
            kerr_attn.bwd_host_saved(ctx, sv, h["dout"], h["dq"], h["dk"], h["dv"])

    def step_host_plain():
        for h in hb:
            kerr_attn.fwd_host(ctx, h["q"], h["k"], h["v"], h["o"], h["lse"], H)
        for h in reversed(hb):
            kerr_attn.bwd_host(ctx, h["q"], h["k"], h["v"], h["o"], h["dout"], h["lse"], h["dq"], h["dk"], h["dv"], H)

    def time_host(fn):
        fn()
        sync_all()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            fn()
        sync_all()
        return max_over_ranks(time.perf_counter() - t0) / e2e_steps

    e2e_s = time_host(step_host)
    e2e_plain_s = time_host(step_host_plain)
    for sv in saved:
        sv.close()
    f4 = 4
    h2d = NB * (B * T * 3 * C + B * T * C) * f4
    d2h = NB * ((B * T * C + B * H * T) * f4 + B * T * 3 * C * f4)
    h2d_plain = NB * (B * T * 3 * C * f4 + (B * T * 3 * C + 2 * B * T * C + B * H * T) * f4)

    peaks, peak_src = measured_peaks()
    work = algorithmic(B, T, H, d)
    props = torch.cuda.get_device_properties(dev)
    ck = clocks.summary()
    sm_mhz = ck["sm_mhz"] or peaks.get("sm_max_mhz", 1965.0)
    tensor_path = args.path != "ffma" and d == 64
    bwd_gbs = work["bwd_bytes"] / (bwd_ms / 1e3) / 1e9
    bwd_tflops = work["bwd_flops"] / (bwd_ms / 1e3) / 1e12
    fwd_tflops = work["fwd_flops"] / (fwd_ms / 1e3) / 1e12
    if tensor_path:
        kernels = ("attn_bwd_rowdot", "attn_bwd_tc64")
        bf16_peak = peaks.get("bf16_tflops")
        # Executed on the tensor pipe per query tile: S^T recomputed, dP^T, dV and
        # dK at 3 MMAs each (bf16 hi/lo split), dQ as two stacked M=128 MMAs
        # (the work of 4): 16 products' worth against the 4 algorithmic ones.
        pipe = {"name": "tcgen05 kind::f16 (bf16 hi/lo split; S^T recomputed)",
                "achieved_tflops": bwd_tflops, "executed_tflops": 4 * bwd_tflops,
                "peak_tflops": bf16_peak, "frac": (4 * bwd_tflops / bf16_peak) if bf16_peak else None,
                "peak_source": f"{peak_src} dense bf16 (burst)",
                "algorithmic_flops_per_launch": work["bwd_flops"]}
    else:
        kernels = ("attn_bwd_rowdot", "attn_bwd_f32")
        ffma_peak_tflops = props.multi_processor_count * 128 * 2 * sm_mhz * 1e6 / 1e12
        pipe = {"name": "fp32 FFMA (CUDA cores)", "achieved_tflops": bwd_tflops,
                "peak_tflops": ffma_peak_tflops, "frac": bwd_tflops / ffma_peak_tflops,
                "peak_source": "nominal: SMs x 128 FMA/clk x 2 x median sampled SM clock",
                "algorithmic_flops_per_launch": work["bwd_flops"]}
    traffic = profiled_traffic(*kernels)
    fwd_kernel = "attn_fwd_tc64" if tensor_path else "attn_fwd_f32"

    ctx.check_device()
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "value_per_gpu": value / world,
        "value_is": "whole-job tokens/s over all ranks (value_per_gpu: the same divided by n_gpus)",
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded q,k,v ~ N(0,1)/8, dout ~ N(0,1))",
        "config": dict(WORKLOAD, global_batch=B * world, parallelism=f"dp{world}: batch shards; attention itself has no exchange (the sublayer step with its gradient all-reduce is the dp_step record)"),
        "e2e": {"value": tokens_per_step / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "api": "kattn_fwd_host_save + kattn_bwd_host_saved per block (forward state kept on the "
                       "device, as the reference's AttnCache), pinned host buffers"},
        "e2e_plain": {"value": tokens_per_step / e2e_plain_s, "unit": "tokens/s", "h2d_bytes_per_step": h2d_plain,
                      "d2h_bytes_per_step": d2h,
                      "api": "kattn_fwd_host + kattn_bwd_host per block (every input sent up by each call)"},
        "gpu_launches": launches, "kernel_path": args.path,
        "kernel_timing": {"method": "second pass of the same steps with CUDA events around each call",
                          "ms_per_step_with_events": ms_step_ev},
        "roofline": {
            "kernel": f"kattn_bwd call = {kernels[0]} + {kernels[1]} (2 launches), one 768-dim block",
            "bound": "hbm", "achieved": bwd_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": bwd_gbs / peaks["hbm_gbs"], "traffic": traffic, "peak_source": peak_src,
            "algorithmic_bytes_per_launch": work["bwd_bytes"], "launch_ms": bwd_ms,
            "pipe": pipe,
            "fwd": {"kernel": fwd_kernel, "launch_ms": fwd_ms, "achieved_tflops": fwd_tflops,
                    "achieved_gbs": work["fwd_bytes"] / (fwd_ms / 1e3) / 1e9,
                    "frac_hbm": work["fwd_bytes"] / (fwd_ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                    "traffic": profiled_traffic(fwd_kernel),
                    "algorithmic_bytes_per_launch": work["fwd_bytes"]},
        },
        "clocks": ck,
    }
    # The data-parallel step around the path at this world size: the
    # sublayer with its per-block gradient all-reduce, at the 768-dim model
    # and at the 1280-dim model (B=32 per GPU, H=20, T=512), and the
    # long-context configuration sharded across the ranks.  Every rank runs
    # these in the same order (they hold collectives).
    if not args.no_nested:
        n_steps, n_warm = max(3, min(args.steps, 20)), 3
        line["dp_step"] = [
            dp_step_object(ctx, dev, world, rank, 768, 12, 256, 16, 4, n_steps, n_warm, 3000),
            dp_step_object(ctx, dev, world, rank, 1280, 20, 512, 32, 4, n_steps, n_warm, 4000)]
        line["long_context"] = long_context_object(ctx, dev, world, rank, n_steps, n_warm)
        line["block_pipeline"] = block_pipeline_object(ctx, dev, world, rank, n_steps, n_warm)
    if world == 1 and not args.no_cpu_baseline:
        cores = os.cpu_count() or 1
        n_seq = min(cores, B)
        cpu_sample(n_seq, T, H, d)  # warm
        t = cpu_sample(n_seq, T, H, d)
        line["cpu_baseline"] = {
            "value": n_seq * T / (NB * t), "unit": "tokens/s", "cores": n_seq, "kind": "port",
            "sample": f"1 of 4 blocks, {n_seq} of {B} sequences on {n_seq} host threads; scaled to the step"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


LAYER_METRIC = ("attention sublayer (ln_1 + c_attn + causal attention + c_proj) fwd+bwd tokens/s per GPU at "
                "768-dim T=256, sublayer gradients all-reduced over the ranks")


def layer_cpu_sample(n_seq: int, T: int, H: int, d: int, threads: int, seed: int = 11):
    """One block of the sublayer through the oracle (LayerNorm, linear layers,
    attention; forward and backward) over n_seq sequences, the linear and
    attention calls on `threads` host threads."""
    import numpy as np

    from oracle import oracle

    C = H * d
    rng = np.random.default_rng(seed)
    M = n_seq * T
    h = rng.standard_normal((M, C)).astype(np.float32)
    lnw, lnb = np.ones(C, np.float32), np.zeros(C, np.float32)
    wa = rng.uniform(-1, 1, (3 * C, C)).astype(np.float32) / np.sqrt(C)
    wp = rng.uniform(-1, 1, (C, C)).astype(np.float32) / np.sqrt(C)
    ba = np.zeros(3 * C, np.float32)
    bp = np.zeros(C, np.float32)
    dy = rng.standard_normal((M, C)).astype(np.float32)
    t0 = time.perf_counter()
    x = oracle.layernorm_forward(h, lnw, lnb)
    qkv = oracle.linear_forward(x, wa, ba, threads=threads).reshape(n_seq, T, 3 * C)
    q, k, v = qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]
    o, att, _ = oracle.forward(q, k, v, H, threads=threads)
    oracle.linear_forward(o.reshape(M, C), wp, bp, threads=threads)
    d_o = oracle.linear_backward_dx(dy, wp, threads=threads)
    oracle.linear_backward_dw(dy, o.reshape(M, C), threads=threads)
    dq, dk, dv = oracle.backward(d_o.reshape(n_seq, T, C), q, k, v, att, H, threads=threads)
    dqkv = np.concatenate([dq, dk, dv], axis=-1).reshape(M, 3 * C)
    dx = oracle.linear_backward_dx(dqkv, wa, threads=threads)
    oracle.linear_backward_dw(dqkv, x, threads=threads)
    oracle.layernorm_backward(dx, h, lnw)
    return time.perf_counter() - t0


def dp_layer_step(ctx, dev, world, C, H, T, B, NB, steps, warmup, seed, exchange=True):
    """Times the data-parallel training step of the attention sublayer on
    this rank: per block LN1, c_attn, attention and c_proj forward, then the
    blocks' backward in reverse order, each block's parameter gradients
    all-reduced across the ranks (NCCL) in two segments, c_proj's as soon as
    its dW is enqueued and the rest when the block's backward is, both
    overlapping the backward still to come (kerr_attn.dist.ProjGradBuckets;
    the reference's host-side gradient sum, src/train.rs:257-269).
    exchange=False skips the all-reduce (the same step on one rank's data
    alone).  Returns the step time (max over ranks) and what it moved."""
    import torch

    import kerr_attn
    from kerr_attn.dist import ProjGradBuckets
    from kerr_attn.dist import max_over_ranks as _max_over_ranks
    from kerr_attn.dist import sync as _sync

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    blocks = []
    for _ in range(NB):
        # LayerNorm init weight 1, bias 0; linear init U(+-1/sqrt(fan_in)),
        # bias 0 (src/init.rs:9-23).
        blk = {"h": torch.randn(B, T, C, device=dev, generator=g),
               "lnw": torch.ones(C, device=dev), "lnb": torch.zeros(C, device=dev),
               "x": torch.empty(B, T, C, device=dev), "dh": torch.empty(B, T, C, device=dev),
               "wa": (torch.rand(3 * C, C, device=dev, generator=g) * 2 - 1) / math.sqrt(C),
               "ba": torch.zeros(3 * C, device=dev),
               "wp": (torch.rand(C, C, device=dev, generator=g) * 2 - 1) / math.sqrt(C),
               "bp": torch.zeros(C, device=dev),
               "qkv": torch.empty(B, T, 3 * C, device=dev), "o": torch.empty(B, T, C, device=dev),
               "lse": torch.empty(B, H, T, device=dev), "y": torch.empty(B, T, C, device=dev),
               "dy": torch.randn(B, T, C, device=dev, generator=g), "d_o": torch.empty(B, T, C, device=dev),
               "dqkv": torch.empty(B, T, 3 * C, device=dev), "dx": torch.empty(B, T, C, device=dev)}
        blk["q"], blk["k"], blk["v"] = kerr_attn.split_qkv(blk["qkv"], C)
        blk["dq"], blk["dk"], blk["dv"] = kerr_attn.split_qkv(blk["dqkv"], C)
        blocks.append(blk)
    buckets = ProjGradBuckets(NB, C, B, device=dev)

    def step():
        n = 0
        for b in blocks:
            n += kerr_attn.layernorm_fwd(ctx, b["h"], b["lnw"], b["lnb"], b["x"])
            n += kerr_attn.linear_fwd(ctx, b["x"], b["wa"], b["ba"], b["qkv"])
            n += kerr_attn.fwd(ctx, b["q"], b["k"], b["v"], b["o"], b["lse"], H)
            n += kerr_attn.linear_fwd(ctx, b["o"], b["wp"], b["bp"], b["y"])
        for i in reversed(range(NB)):
            b = blocks[i]
            aw, ab, pw, pb = buckets.views(i)
            n += kerr_attn.linear_bwd_dx(ctx, b["dy"], b["wp"], b["d_o"])
            n += kerr_attn.linear_bwd_dw(ctx, b["dy"], b["o"], pw, pb, accumulate=False)
            if exchange:
                buckets.launch_proj(i)
            n += kerr_attn.bwd(ctx, b["q"], b["k"], b["v"], b["o"], b["d_o"], b["lse"], b["dq"], b["dk"], b["dv"], H)
            n += kerr_attn.linear_bwd_dx(ctx, b["dqkv"], b["wa"], b["dx"])
            n += kerr_attn.linear_bwd_dw(ctx, b["dqkv"], b["x"], aw, ab, accumulate=False)
            lw, lb = buckets.ln_views(i)
            n += kerr_attn.layernorm_bwd(ctx, b["dx"], b["h"], b["lnw"], b["dh"], lw, lb, accumulate=False)
            if exchange:
                buckets.launch(i)
        buckets.finish()
        return n

    for _ in range(warmup):
        step()
    _sync(dev)
    mk = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    t0, t1 = mk(), mk()
    _sync(dev)
    t0.record()
    launches = 0
    for _ in range(steps):
        launches += step()
    t1.record()
    torch.cuda.synchronize(dev)
    _sync(dev)
    ms_step = _max_over_ranks(t0.elapsed_time(t1), dev) / steps
    del blocks
    return {"ms_per_step": ms_step, "tokens_per_s": B * T * world / (ms_step / 1e3), "steps": steps,
            "gpu_launches": launches,
            "allreduce": {"segments_per_step": 2 * NB if (exchange and world > 1) else 0,
                          "bytes_per_step": NB * buckets.numel * 4 if (exchange and world > 1) else 0,
                          "backend": "nccl" if (exchange and world > 1) else "none"}}


def dp_step_object(ctx, dev, world, rank, C, H, T, B, NB, steps, warmup, seed):
    """The nested record of one data-parallel sublayer configuration: the
    step with its gradient all-reduce, the same step without the exchange,
    and the ratio of the two (the exchange's cost at this world size)."""
    import torch

    full = dp_layer_step(ctx, dev, world, C, H, T, B, NB, steps, warmup, seed + rank, exchange=True)
    torch.cuda.empty_cache()
    alone = dp_layer_step(ctx, dev, world, C, H, T, B, NB, steps, warmup, seed + rank, exchange=False)
    torch.cuda.empty_cache()
    d = C // H
    work = algorithmic(B, T, H, d)
    flops = NB * (24.0 * B * T * C * C + work["fwd_flops"] + work["bwd_flops"])
    return {"workload": f"attention sublayer (ln_1, c_attn, causal attention, c_proj) fwd+bwd, n_embd {C}, "
                        f"{H} heads, seq_len {T}, {B} sequences per GPU, {NB} blocks",
            "n_gpus": world, "global_batch": B * world, **full,
            "ms_per_step_without_exchange": alone["ms_per_step"],
            "efficiency_vs_no_exchange": alone["ms_per_step"] / full["ms_per_step"],
            "algorithmic_tflops": flops / (full["ms_per_step"] / 1e3) / 1e12}


def block_pipeline_object(ctx, dev, world, rank, steps, warmup, C=768, H=12, T=256, B=16, NB=4, rk4=8):
    """The device-resident block pipeline (kattn_block_*): the 768-dim
    model's 4 blocks, each LN1, c_attn, attention, c_proj and the residual,
    then LN2 and the Kerr-ODE FFN core (rk4_n_steps 8) with its residual,
    forward through the blocks and backward in reverse, two C-ABI calls per
    block with every intermediate on the device (the reference's
    forward_backward_batch, src/pipeline.rs:764-1222, without the FFN's dense
    maestro layers).  Each rank runs its own 16 sequences: no exchange."""
    import torch

    import kerr_attn
    from kerr_attn.dist import max_over_ranks as _max_over_ranks
    from kerr_attn.dist import sync as _sync

    g = torch.Generator(device=dev)
    g.manual_seed(5000 + rank)
    nb = C // 2

    def lin(n_out, n_in):
        return (torch.rand(n_out, n_in, device=dev, generator=g) * 2 - 1) / math.sqrt(n_in), \
            torch.zeros(n_out, device=dev)

    params, grads, blocks = [], [], []
    for _ in range(NB):
        wa, ba = lin(3 * C, C)
        wp, bp = lin(C, C)
        P = {"ln1_w": torch.ones(C, device=dev), "ln1_b": torch.zeros(C, device=dev), "w_attn": wa, "b_attn": ba,
             "w_proj": wp, "b_proj": bp, "ln2_w": torch.ones(C, device=dev), "ln2_b": torch.zeros(C, device=dev),
             "gamma_raw": torch.full((nb,), math.log(math.expm1(0.1)), device=dev),
             "omega": (torch.arange(nb, device=dev, dtype=torch.float32) + 1) / nb,
             "alpha_beta": torch.tensor([0.1, 0.1], device=dev)}
        params.append(P)
        grads.append({k: torch.empty_like(v) for k, v in P.items()})
        blocks.append(kerr_attn.Block(ctx, B, T, C, H, rk4))
    hs = [torch.randn(B, T, C, device=dev, generator=g)] + [torch.empty(B, T, C, device=dev) for _ in range(NB)]
    dy = torch.randn(B, T, C, device=dev, generator=g)
    dh = torch.empty(B, T, C, device=dev)

    def step():
        n = 0
        for i in range(NB):
            n += blocks[i].fwd(params[i], hs[i], hs[i + 1])
        src = dy
        for i in reversed(range(NB)):
            n += blocks[i].bwd(src, dh, grads[i])
            src = dh
        return n

    for _ in range(warmup):
        step()
    _sync(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    launches = 0
    for _ in range(steps):
        launches += step()
    t1.record()
    torch.cuda.synchronize(dev)
    _sync(dev)
    ms = _max_over_ranks(t0.elapsed_time(t1), dev) / steps
    for b in blocks:
        b.close()
    del hs, params, grads
    torch.cuda.empty_cache()
    return {"workload": f"device-resident block pipeline (kattn_block_fwd / _bwd): n_embd {C}, {H} heads, "
                        f"seq_len {T}, {B} sequences per GPU, {NB} blocks of LN1, c_attn, causal attention, "
                        f"c_proj, LN2 and the Kerr-ODE FFN core (rk4_n_steps {rk4}) with residuals, fwd+bwd",
            "n_gpus": world, "ms_per_step": ms, "tokens_per_s": B * T * world / (ms / 1e3), "steps": steps,
            "gpu_launches": launches, "exchange": "none (independent sequences per rank)"}


LONG_CONTEXT = {"batch": 8, "n_head": 12, "head_dim": 64, "seq_lens": (1024, 2048, 4096)}


def long_context_object(ctx, dev, world, rank, steps, warmup):
    """The long-context configuration (B=8, H=12, d=64, T = 1024, 2048,
    4096; q, k, v ~ N(0,1)/8, dout ~ N(0,1)) with its 96 (batch, head) slabs
    sharded across the ranks by whole sequences (rank r owns
    shard_batch(8, world, r); no exchange).  Per T: fwd+bwd time (max over
    ranks), whole-job tokens/s and the fraction of this GPU's roofline for
    the shard it ran (the larger of its HBM bytes at the measured copy rate
    and its tensor-core flops, 3 bf16 MMAs per product, at the measured bf16
    rate)."""
    import torch

    import kerr_attn
    from kerr_attn.dist import max_over_ranks as _max_over_ranks
    from kerr_attn.dist import shard_batch
    from kerr_attn.dist import sync as _sync

    L = LONG_CONTEXT
    H, d = L["n_head"], L["head_dim"]
    C = H * d
    b0, b1 = shard_batch(L["batch"], world, rank)
    nb = b1 - b0
    peaks, peak_src = measured_peaks()
    hbm = peaks.get("hbm_gbs", FALLBACK_HBM_GBS)
    bf16 = peaks.get("bf16_tflops") or 1590.0
    stream = torch.cuda.current_stream(dev)
    out = []
    for T in L["seq_lens"]:
        g = torch.Generator(device=dev)
        g.manual_seed(5000 + T + 17 * rank)
        per_set = 4 * max(nb, 1) * T * 9 * C
        nbuf = max(1, math.ceil(256e6 / per_set))  # rotate distinct buffers: > L2 per round
        bufs = []
        for _ in range(nbuf if nb else 0):
            qkv = torch.randn(nb, T, 3 * C, device=dev, generator=g) / 8
            b = {"qkv": qkv, "o": torch.empty(nb, T, C, device=dev), "lse": torch.empty(nb, H, T, device=dev),
                 "dout": torch.randn(nb, T, C, device=dev, generator=g), "dqkv": torch.empty_like(qkv)}
            b["q"], b["k"], b["v"] = kerr_attn.split_qkv(b["qkv"], C)
            b["dq"], b["dk"], b["dv"] = kerr_attn.split_qkv(b["dqkv"], C)
            bufs.append(b)

        def one(i):
            if not bufs:
                return 0
            b = bufs[i % len(bufs)]
            n = kerr_attn.fwd(ctx, b["q"], b["k"], b["v"], b["o"], b["lse"], H, stream=stream)
            return n + kerr_attn.bwd(ctx, b["q"], b["k"], b["v"], b["o"], b["dout"], b["lse"], b["dq"], b["dk"],
                                     b["dv"], H, stream=stream)

        for i in range(warmup):
            one(i)
        reps = max(nbuf, steps)
        _sync(dev)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        launches = 0
        for i in range(reps):
            launches += one(i)
        t1.record(stream)
        torch.cuda.synchronize(dev)
        _sync(dev)
        ms = _max_over_ranks(t0.elapsed_time(t1) / reps, dev)
        w = algorithmic(max(nb, 1), T, H, d)
        byts = w["fwd_bytes"] + w["bwd_bytes"]
        flops = w["fwd_flops"] + w["bwd_flops"]
        t_roof_ms = 1e3 * max(byts / (hbm * 1e9), 3 * flops / (bf16 * 1e12))
        out.append({"seq_len": T, "sequences_per_gpu": nb, "slabs_per_gpu": nb * H, "ms_per_step": ms,
                    "tokens_per_s": L["batch"] * T / (ms / 1e3), "steps": reps, "gpu_launches": launches,
                    "roofline_frac": t_roof_ms / ms, "roofline_ms": t_roof_ms,
                    "bound": "tensor" if 3 * flops / (bf16 * 1e12) > byts / (hbm * 1e9) else "hbm",
                    "algorithmic_tflops": flops / (ms / 1e3) / 1e12,
                    "l2": f"{nbuf} distinct buffer sets rotated" if nbuf > 1 else "inputs exceed L2"})
        del bufs
        torch.cuda.empty_cache()
    return {"workload": "long-context causal attention fwd+bwd, B=8, H=12, d=64, 96 (batch, head) slabs sharded "
                        "by whole sequences across the ranks, no exchange",
            "peaks": f"HBM {hbm} GB/s, bf16 {bf16} TF/s ({peak_src})", "per_seq_len": out}


def run_layer(args):
    """The whole attention sublayer of the 768-dim model per block
    (src/pipeline.rs:236-249) as the data-parallel step of dp_layer_step:
    LN1, c_attn, attention, c_proj forward; their backward in reverse block
    order; each block's parameter gradients (c_attn, c_proj, ln_1) all-reduced
    across the ranks (NCCL) while the blocks below run their backward."""
    import torch
    import torch.distributed as dist

    import kerr_attn
    from kerr_attn.dist import world as _world

    rank, local, world = _world()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 under torchrun")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    W = WORKLOAD
    B, T, H, d, NB = W["batch_per_gpu"], W["seq_len"], W["n_head"], W["head_dim"], W["blocks"]
    C = H * d
    M = B * T
    ctx = kerr_attn.Context(local)
    clocks = ClockSampler(local)
    clocks.start()
    r = dp_layer_step(ctx, dev, world, C, H, T, B, NB, args.steps, args.warmup, 2000 + rank)
    clocks.stop()
    ms_step = r["ms_per_step"]
    tokens = B * T * world
    work = algorithmic(B, T, H, d)
    gemm_flops = 24.0 * M * C * C  # c_attn and c_proj: forward, dx and dW (2 flops per MAC)
    attn_flops = work["fwd_flops"] + work["bwd_flops"]
    flops_step = NB * (gemm_flops + attn_flops)
    achieved = flops_step / (ms_step / 1e3) / 1e12
    peaks, peak_src = measured_peaks()
    bf16 = peaks.get("bf16_tflops_sustained") or peaks.get("bf16_tflops")
    ctx.check_device()
    line = {"metric": LAYER_METRIC, "value": tokens / (ms_step / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded h, dy ~ N(0,1); LayerNorm init 1 / 0; linear init U(+-1/sqrt(fan_in)), "
                    "bias 0)",
            "config": dict(W, workload="kerr-engine 768-dim attention sublayer fwd+bwd (ln_1, c_attn, attention, "
                                       "c_proj), 4 blocks per step", global_batch=B * world,
                           parallelism=f"dp{world}, sublayer parameter gradients all-reduced per block"),
            "gpu_launches": r["gpu_launches"],
            "allreduce": r["allreduce"],
            "roofline": {"bound": "tensor", "achieved": achieved, "unit": "TFLOP/s",
                         "algorithmic_flops_per_step": flops_step,
                         "executed_tflops": 3 * achieved, "peak": bf16,
                         "frac": (3 * achieved / bf16) if bf16 else None,
                         "peak_source": f"{peak_src} dense bf16 (sustained)",
                         "note": "every product runs as 3 bf16 MMAs (hi/lo split): executed = 3 x algorithmic"},
            "clocks": clocks.summary()}
    if world == 1 and not args.no_cpu_baseline:
        cores = os.cpu_count() or 1
        n_seq = min(4, B)
        layer_cpu_sample(n_seq, T, H, d, cores)
        t = layer_cpu_sample(n_seq, T, H, d, cores)
        line["cpu_baseline"] = {"value": n_seq * T / (NB * t), "unit": "tokens/s", "cores": cores, "kind": "port",
                                "sample": f"1 of 4 blocks, {n_seq} of {B} sequences, every oracle call on "
                                          f"{cores} host threads; scaled to the 4-block step"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


KERR_METRIC = "Kerr-ODE (FFN ODE core) fwd+bwd tokens/s per GPU at 768-dim T=256, 4 blocks; % of FP32 roofline"
KERR = {"workload": "kerr-engine 768-dim Kerr-ODE fwd+bwd (rk4_n_steps 8), 4 blocks per step",
        "batch_per_gpu": 16, "seq_len": 256, "n_embd": 768, "n_bands": 384, "rk4_n_steps": 8, "blocks": 4,
        "layout": "rows of n_embd floats, bands interleaved (r, s)",
        "l2": "no flush: 4 blocks x 50 MB of distinct x, y, dy, dx buffers per step exceed the 126 MB L2"}


def kerr_algorithmic(M, nb, n_steps):
    """Floating-point operations of the reference's formulas per launch
    (src/model.rs:778-843; src/backward.rs:184-379), counted per band and RK4
    step: forward 90 (4 derivative evaluations of 16, three intermediate
    states of 4, the weighted combination of 14); backward 300 (the step's
    forward again, the fourth evaluation's stencil, four adjoint evaluations of
    29 and their chaining).  Bytes: forward reads x and writes y, backward
    reads dy and x and writes dx (4 bytes per float, 2 floats per band)."""
    units = M * nb
    return {"fwd_flops": 90.0 * n_steps * units, "bwd_flops": 300.0 * n_steps * units,
            "fwd_bytes": 16.0 * units, "bwd_bytes": 24.0 * units}


def run_kerr(args):
    """Kerr-ODE of the 768-dim model: each block's forward, then the backwards
    in reverse block order (the FFN's ODE calls of one training step,
    src/pipeline.rs:1067, :1107).  Weak scaling: every rank runs its own
    16 sequences; the parameter gradients are per-rank sums (the data-parallel
    reduction of the FFN parameters is outside this path)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    import kerr_attn
    from kerr_attn.dist import max_over_ranks as _max_over_ranks
    from kerr_attn.dist import sync as _sync
    from kerr_attn.dist import world as _world

    rank, local, world = _world()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 under torchrun")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    K = KERR
    B, T, nb, n_steps, NB = K["batch_per_gpu"], K["seq_len"], K["n_bands"], K["rk4_n_steps"], K["blocks"]
    M, n = B * T, 2 * nb
    ctx = kerr_attn.Context(local)
    g = torch.Generator(device=dev)
    g.manual_seed(3000 + rank)
    # The reference's initial KerrWeights (src/init.rs:50-61); inputs ~ N(0,1)
    # as LN2's output (plus the input maestro's small correction) is.
    gamma_raw = torch.full((nb,), math.log(math.expm1(0.1)), device=dev)
    omega = (torch.arange(nb, device=dev, dtype=torch.float32) + 1) / nb
    ab = torch.tensor([0.1, 0.1], device=dev)
    blocks = [{"x": torch.randn(M, n, device=dev, generator=g), "y": torch.empty(M, n, device=dev),
               "dy": torch.randn(M, n, device=dev, generator=g), "dx": torch.empty(M, n, device=dev),
               "dg": torch.zeros(nb, device=dev), "do": torch.zeros(nb, device=dev),
               "dab": torch.zeros(2, device=dev)} for _ in range(NB)]
    stream = torch.cuda.current_stream(dev)

    def step(ev=None):
        c = 0
        for i, b in enumerate(blocks):
            if ev is not None:
                ev["f"][i][0].record(stream)
            c += kerr_attn.kerr_ode_fwd(ctx, b["x"], gamma_raw, omega, ab, b["y"], n_steps, stream=stream)
            if ev is not None:
                ev["f"][i][1].record(stream)
        for i in reversed(range(NB)):
            b = blocks[i]
            if ev is not None:
                ev["b"][i][0].record(stream)
            c += kerr_attn.kerr_ode_bwd(ctx, b["dy"], b["x"], gamma_raw, omega, ab, b["dx"], b["dg"], b["do"],
                                        b["dab"], n_steps, accumulate=False, stream=stream)
            if ev is not None:
                ev["b"][i][1].record(stream)
        return c

    for _ in range(args.warmup):
        step()
    _sync(dev)
    mk = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    clocks = ClockSampler(local)
    clocks.start()
    t0, t1 = mk(), mk()
    _sync(dev)
    t0.record(stream)
    launches = 0
    for _ in range(args.steps):
        launches += step()
    t1.record(stream)
    torch.cuda.synchronize(dev)
    clocks.stop()
    _sync(dev)
    ms_step = _max_over_ranks(t0.elapsed_time(t1), dev) / args.steps
    evs = [{"f": [(mk(), mk()) for _ in range(NB)], "b": [(mk(), mk()) for _ in range(NB)]}
           for _ in range(args.steps)]
    _sync(dev)
    for s_ in range(args.steps):
        step(evs[s_])
    torch.cuda.synchronize(dev)
    _sync(dev)
    fwd_ms = _max_over_ranks(statistics.mean(e["f"][i][0].elapsed_time(e["f"][i][1]) for e in evs
                                             for i in range(NB)), dev)
    bwd_ms = _max_over_ranks(statistics.mean(e["b"][i][0].elapsed_time(e["b"][i][1]) for e in evs
                                             for i in range(NB)), dev)
    work = kerr_algorithmic(M, nb, n_steps)
    ck = clocks.summary()
    peaks, peak_src = measured_peaks()
    props = torch.cuda.get_device_properties(dev)
    sm_mhz = ck["sm_mhz"] or peaks.get("sm_max_mhz", 1965.0)
    fp32_peak = props.multi_processor_count * 128 * 2 * sm_mhz * 1e6 / 1e12
    hbm = peaks.get("hbm_gbs", FALLBACK_HBM_GBS)
    fwd_tf = work["fwd_flops"] / (fwd_ms / 1e3) / 1e12
    bwd_tf = work["bwd_flops"] / (bwd_ms / 1e3) / 1e12
    ctx.check_device()

    # End to end through the host-buffer ABI (kattn_kerr_ode_fwd_host /
    # _bwd_host, the trait's host-slice boundary): pinned host x, dy and
    # KerrWeights in; y, dx and the parameter gradients out, every call.
    hx = [b["x"].cpu().pin_memory() for b in blocks]
    hdy = [b["dy"].cpu().pin_memory() for b in blocks]
    hy = [torch.empty(M, n).pin_memory() for _ in blocks]
    hdx = [torch.empty(M, n).pin_memory() for _ in blocks]
    hg, ho = gamma_raw.cpu(), omega.cpu()
    hpar = [(torch.empty(nb), torch.empty(nb), torch.empty(2)) for _ in blocks]

    def step_e2e():
        for i in range(NB):
            kerr_attn.kerr_ode_fwd_host(ctx, hx[i], hg, ho, 0.1, 0.1, hy[i], n_steps)
        for i in reversed(range(NB)):
            kerr_attn.kerr_ode_bwd_host(ctx, hdy[i], hx[i], hg, ho, 0.1, 0.1, hdx[i], *hpar[i], n_steps,
                                        accumulate=False)

    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    step_e2e()
    _sync(dev)
    e0, e1 = mk(), mk()
    e0.record(stream)
    for _ in range(e2e_steps):
        step_e2e()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    _sync(dev)
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1), dev) / e2e_steps
    tokens = B * T * world
    line = {"metric": KERR_METRIC, "value": tokens / (ms_step / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded x, dy ~ N(0,1); the reference's initial KerrWeights)",
            "config": dict(K, global_batch=B * world, parallelism=f"dp{world} (positions sharded, no exchange)"),
            "e2e": {"value": tokens / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": NB * (3 * M * n + 2 * (2 * nb + 2)) * 4,
                    "d2h_bytes_per_step": NB * (2 * M * n + 2 * nb + 2) * 4,
                    "api": "kattn_kerr_ode_fwd_host / _bwd_host per block (synchronous host-buffer calls): pinned "
                           "x (twice) and dy up, y, dx and the parameter gradients down"},
            "gpu_launches": launches,
            "roofline": {"kernel": "kode_bwd + kode_param_final (one kattn_kerr_ode_bwd call, one block)",
                         "bound": "fp32", "achieved": bwd_tf, "peak": fp32_peak, "unit": "TFLOP/s",
                         "frac": bwd_tf / fp32_peak, "launch_ms": bwd_ms,
                         "algorithmic_flops_per_launch": work["bwd_flops"],
                         "traffic": profiled_traffic("kode_bwd"),
                         "peak_source": f"nominal FP32 FMA rate (148 SMs x 128 lanes x 2) at the sampled "
                                        f"{sm_mhz:.0f} MHz; not in MEASURED_PEAKS.json",
                         "hbm": {"achieved_gbs": work["bwd_bytes"] / (bwd_ms / 1e3) / 1e9, "peak_gbs": hbm,
                                 "frac": work["bwd_bytes"] / (bwd_ms / 1e3) / 1e9 / hbm,
                                 "peak_source": peak_src},
                         "fwd": {"kernel": "kode_fwd", "launch_ms": fwd_ms, "achieved_tflops": fwd_tf,
                                 "frac": fwd_tf / fp32_peak,
                                 "achieved_gbs": work["fwd_bytes"] / (fwd_ms / 1e3) / 1e9}},
            "clocks": ck}
    if world == 1 and not args.no_cpu_baseline:
        from oracle import oracle

        oracle.build()
        cores = os.cpu_count() or 1
        m = 16 * cores
        rng = np.random.default_rng(5)
        x = rng.standard_normal((m, n)).astype(np.float32)
        dy = rng.standard_normal((m, n)).astype(np.float32)
        gr, om = gamma_raw.cpu().numpy(), omega.cpu().numpy()
        t_0 = time.perf_counter()
        oracle.kerr_ode_forward(x, gr, om, 0.1, 0.1, n_steps, threads=cores)
        oracle.kerr_ode_backward(dy, x, gr, om, 0.1, 0.1, n_steps, threads=cores)
        t = time.perf_counter() - t_0
        line["cpu_baseline"] = {"value": m / (NB * t), "unit": "tokens/s", "cores": cores, "kind": "port",
                                "sample": f"1 of 4 blocks, {m} of {M} positions (fwd + bwd) on {cores} host "
                                          f"threads; scaled to the 4-block step"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


SWEEP_METRIC = "causal-attn fwd+bwd tokens/s and % of roofline per configuration (one GPU)"


def run_sweep(args):
    """The attention configurations besides the headline, each timed alone on
    one GPU: the d=32 microbenchmark (B=64, H=4, T=256, q,k,v ~ N(0,1)/sqrt(32))
    and the long-context sweep (B=8, H=12, d=64, T = 1024, 2048, 4096,
    q,k,v ~ N(0,1)/8); dout ~ N(0,1).  One line per configuration, with the
    achieved HBM GB/s and TFLOP/s of the fwd+bwd pair against the measured
    peaks (the long-context sweep shards 96 slabs across GPUs with no
    exchange; one GPU runs all of them here)."""
    import torch

    import kerr_attn

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ctx = kerr_attn.Context(0)
    ctx.set_path({"auto": kerr_attn.PATH_AUTO, "ffma": kerr_attn.PATH_FFMA, "tensor": kerr_attn.PATH_TENSOR}[args.path])
    peaks, peak_src = measured_peaks()
    hbm = peaks.get("hbm_gbs", FALLBACK_HBM_GBS)
    bf16 = peaks.get("bf16_tflops")
    props = torch.cuda.get_device_properties(dev)
    mk = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    stream = torch.cuda.current_stream(dev)
    configs = (("d32", "attention microbenchmark d=32", 64, 4, 256, 32, 1 / math.sqrt(32)),
               ("t1024", "long-context T=1024", 8, 12, 1024, 64, 1 / 8),
               ("t2048", "long-context T=2048", 8, 12, 2048, 64, 1 / 8),
               ("t4096", "long-context T=4096", 8, 12, 4096, 64, 1 / 8))
    only = set(args.sweep_only.split(",")) if args.sweep_only else None
    for key, name, B, H, T, d, sig in configs:
        if only is not None and key not in only:
            continue
        C = H * d
        g = torch.Generator(device=dev)
        g.manual_seed(B * T + d)
        nbuf = max(1, math.ceil(256e6 / (4 * B * T * 9 * C)))  # distinct buffers: > L2 per round
        bufs = []
        for _ in range(nbuf):
            qkv = torch.randn(B, T, 3 * C, device=dev, generator=g) * sig
            b = {"qkv": qkv, "o": torch.empty(B, T, C, device=dev), "lse": torch.empty(B, H, T, device=dev),
                 "dout": torch.randn(B, T, C, device=dev, generator=g), "dqkv": torch.empty_like(qkv)}
            b["q"], b["k"], b["v"] = kerr_attn.split_qkv(b["qkv"], C)
            b["dq"], b["dk"], b["dv"] = kerr_attn.split_qkv(b["dqkv"], C)
            bufs.append(b)

        def one(b):
            c = kerr_attn.fwd(ctx, b["q"], b["k"], b["v"], b["o"], b["lse"], H, stream=stream)
            return c + kerr_attn.bwd(ctx, b["q"], b["k"], b["v"], b["o"], b["dout"], b["lse"], b["dq"], b["dk"],
                                     b["dv"], H, stream=stream)

        for i in range(max(3, args.warmup)):
            one(bufs[i % nbuf])
        torch.cuda.synchronize(dev)
        reps = max(nbuf, min(args.steps, 40 if T <= 1024 else 10))
        clocks = ClockSampler(0)
        clocks.start()
        t0, t1 = mk(), mk()
        t0.record(stream)
        launches = 0
        for i in range(reps):
            launches += one(bufs[i % nbuf])
        t1.record(stream)
        torch.cuda.synchronize(dev)
        clocks.stop()
        ms = t0.elapsed_time(t1) / reps
        w = algorithmic(B, T, H, d)
        flops = w["fwd_flops"] + w["bwd_flops"]
        byts = w["fwd_bytes"] + w["bwd_bytes"]
        tf = flops / (ms / 1e3) / 1e12
        gbs = byts / (ms / 1e3) / 1e9
        ck = clocks.summary()
        sm_mhz = ck["sm_mhz"] or peaks.get("sm_max_mhz", 1965.0)
        # The kernel family the library picks: tensor cores at d=64, and at d=32
        # from 16384 (batch, head, position) rows up (AUTO), or as asked.
        tensor = args.path != "ffma" and (d == 64 or (d == 32 and (args.path == "tensor" or B * H * T >= 16384)))
        # Roofline time: HBM bytes at the measured copy rate, or the pipe's
        # executed flops at its peak (tensor path: 3 MMAs per forward product;
        # 4x the backward's algorithmic flops, S^T recomputed and dQ stacked).
        pipe_tflops = bf16 if tensor else props.multi_processor_count * 256 * sm_mhz * 1e-6
        executed = (3 * w["fwd_flops"] + 4 * w["bwd_flops"]) if tensor else flops
        t_roof = max(byts / (hbm * 1e9), executed / (pipe_tflops * 1e12))
        line = {"metric": SWEEP_METRIC, "value": B * T / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
                "steps": reps, "ms_per_step": ms, "higher_is_better": True, "dtype": "f32",
                "data": f"synthetic (seeded q,k,v ~ N(0,1) x {sig:.4f}, dout ~ N(0,1))",
                "config": {"workload": name, "batch": B, "n_head": H, "seq_len": T, "head_dim": d, "causal": True,
                           "l2": f"{nbuf} distinct buffer sets rotated" if nbuf > 1 else "inputs exceed L2"},
                "kernel_path": "tcgen05 bf16x3" if tensor else "fp32 FFMA",
                "gpu_launches": launches,
                "roofline": {"achieved_gbs": gbs, "hbm_peak_gbs": hbm, "hbm_frac": gbs / hbm,
                             "achieved_tflops": tf, "frac_of_roofline": (t_roof * 1e3) / ms,
                             "roofline_ms": t_roof * 1e3,
                             "pipe": ("tcgen05 kind::f16, 3 MMAs per product, measured dense bf16 "
                                      f"{bf16} TF/s ({peak_src})") if tensor else
                                     f"FP32 FFMA nominal at {sm_mhz:.0f} MHz",
                             "pipe_frac": executed / (ms / 1e3) / 1e12 / pipe_tflops},
                "clocks": ck}
        print(json.dumps(line), flush=True)
        del bufs
        torch.cuda.empty_cache()
    ctx.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sweep-only", default="",
                    help="--workload sweep: comma-separated subset of d32, t1024, t2048, t4096")
    ap.add_argument("--no-nested", action="store_true",
                    help="skip the nested data-parallel step and long-context records of the headline line")
    ap.add_argument("--path", choices=("auto", "ffma", "tensor"), default="auto",
                    help="kernel family (auto: tensor cores where supported)")
    ap.add_argument("--workload", choices=("attention", "layer", "kerr", "sweep"), default="attention",
                    help="attention: the headline (attention fwd+bwd); layer: c_attn + attention + c_proj with "
                         "the projection-gradient all-reduce; kerr: the Kerr-ODE fwd+bwd; sweep: the d=32 "
                         "microbenchmark and the long-context configurations, one line each")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "layer":
        run_layer(args)
    elif args.workload == "kerr":
        run_kerr(args)
    elif args.workload == "sweep":
        run_sweep(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
