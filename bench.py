#!/usr/bin/env python3
"""Benchmark of the B200 speculative-decoding path.

Workload ("int8"): decoder with 4 layers, d_model 256,
4 heads x 64, FFN 1024, vocab 2048; target weights int8 per output channel,
fp32 activations and KV cache; draft = the target's first layer + shared
lm_head; per GPU 8 requests with 64-token uniform-random prompts,
temperature 1.0 rejection sampling, k = 4, 256 new tokens, Philox uniforms
from the host.  Architecture: the reference TransformerDecoder (post-LN,
SwiGLU, RoPE; --arch cfg selects the pre-LN/GELU/learned-position variant).
Weights are seeded synthetic (no checkpoints exist for this path).

One step = one generate call over the GPU's batch: prefill of target and
draft, then speculative rounds until every request has 256 new tokens.
`value` is new tokens per second over all GPUs with prompts already resident
in HBM; `e2e` is the same metric through the public C ABI with host buffers
(prompt + uniform upload and token download inside the timed region).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Multi-GPU: launch with torchrun; requests are partitioned by rank (weak
scaling, no data-path collective); timing is the max over ranks.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "neural-network_b200"))

from specdec_b200.synth import (ARCH_CFG, ARCH_REF, device_params, draft_params, make_params,  # noqa: E402
                                 make_prompts, workload)

METRIC = "accepted tokens/sec per GPU (spec-decode, k=4) at 1/2/4/8 B200; % HBM roofline"
UNIT = "tokens/s"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d.get("hbm_gbs", 6650.0)), "measured"
    return 6650.0, "fallback"


def bf16_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f).get("bf16_tflops", 1590.0))
    return 1590.0


def tree_nodes(branching) -> int:
    n, level = 0, 1
    for b in branching:
        level *= b
        n += level
    return n


KV_DTYPE = {0: 0, 1: 1, 2: 2}  # workload kv_mode -> SPECDEC_F32 / BF16 / INT8

# The large workload at one GPU's share of its 256
# requests when they are split over 8 GPUs.
LARGE_REQUESTS_PER_GPU = 32


# DRAM bytes (read + write) of one launch of the roofline kernel, from the ncu
# capture named beside it (caches flushed before the launch, as the live probe
# does); None where no capture of the current kernel exists.
TRAFFIC = {
    "int8": (503808, "profiles/linear_resid_int8_verify_dram.md"),
}


def roofline_entry(p, hbm, tflops, wl, rows):
    """The FFN down-projection at the verify row count: HBM-bound below the
    bf16 ridge (peak flops / peak bytes), tensor-bound above it."""
    ridge = tflops * 1e12 / (hbm * 1e9)
    what = "tcgen05 GEMM" if (wl.act_bf16 and rows >= 64) else "linear_kernel GEMV"
    kern = f"{what}, residual epilogue (target FFN down-projection, {rows} verify rows)"
    traffic, src = TRAFFIC.get(wl.name, (None, None))
    extra = {"kernel": kern, "traffic_source": src}
    if p["flops_per_byte"] > ridge:
        return {"bound": "tensor", "achieved": p["TFLOPs"], "peak": tflops, "unit": "TFLOP/s",
                "frac": p["TFLOPs"] / tflops, "traffic": traffic, **extra}
    return {"bound": "hbm", "achieved": p["GBps"], "peak": hbm, "unit": "GB/s", "frac": p["GBps"] / hbm,
            "traffic": traffic, **extra}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def algorithmic_bytes_per_round(wl, int8: bool, avg_ctx: float) -> dict:
    """Weight + KV bytes one speculative round must move (k draft steps + verify)."""
    m = wl.target
    d, F, V, L = m.d_model, m.d_ff, m.vocab, m.n_layers
    kvd = m.kv_heads * m.head_dim
    wb = 1 if int8 else 4
    per_layer = (d * (d + 2 * kvd) + d * d + (3 if m.arch == ARCH_REF else 2) * d * F) * wb
    head = d * V * wb
    w_t = L * per_layer + head
    w_d = wl.draft_layers * per_layer + head
    # cache element bytes by KV dtype (f32, bf16, int8 + one fp32 scale per
    # position and kv head for K and for V)
    kv_tok_layer = 2 * kvd * {0: 4, 1: 2, 2: 1}[wl.kv_mode] + (2 * 4 * m.kv_heads if wl.kv_mode == 2 else 0)
    B, k = wl.batch, wl.lookahead
    kv_read = B * avg_ctx * kv_tok_layer * (k * wl.draft_layers + L)
    kv_write = B * kv_tok_layer * ((k + 1) * wl.draft_layers + (k + 1) * L)
    return {"w_target": w_t, "w_draft": w_d, "weights": k * w_d + w_t, "kv": kv_read + kv_write,
            "total": k * w_d + w_t + kv_read + kv_write}


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        self.f.close()

    def summary(self):
        rows = []
        try:
            with open(self.path) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) >= 9:
                        rows.append(parts)
        finally:
            os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def reference_arm(args, wl, rank, world):
    """The reference's own CPU implementation on this host's cores."""
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("gloo", init_method="env://")
    if rank != 0:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return
    if wl.name == "large":
        print(json.dumps({"impl": "reference", "unavailable": "the reference dequantises the large model's 6.6 G "
                          "int8 weights to fp32 (26 GB) on every Dense call; its CPU arm runs on the int8 workload"}),
              flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # the reference arm times the reference (oracle/_ref) or the CPU restatement

    kind = "reference" if oracle.reference_available() else "port"
    ncores = os.cpu_count() or 1
    P = make_params(wl.target, seed=0)
    DP = draft_params(wl.target, P, wl.draft_layers)
    new_per_step = 32 if wl.name == "int8" else 8
    prompts = make_prompts(wl.batch, wl.prompt_len, wl.target.vocab, seed=1)
    if kind == "reference":
        # int8 target: the reference multiplies by the dequantised weight q*s
        # (src/nn/quantization.cpp:127-147); inject those values.
        om = oracle.Oracle(wl.target, P, int8=wl.weights_int8)
        Pq = [om.param(i).reshape(np.shape(P[i])) for i in range(len(P))]
        tgt = oracle.Reference(wl.target, Pq, requires_grad=False)
        dft = oracle.Reference(wl.target.with_layers(wl.draft_layers), draft_params(wl.target, Pq, wl.draft_layers),
                               requires_grad=False)

        def one(i):
            out = tgt.generate_speculative(dft, prompts[i % wl.batch], new_per_step, wl.lookahead,
                                           wl.temperature, 0, 1.0, 1000 + i)
            return len(out) - wl.prompt_len
    else:
        tgt = oracle.Oracle(wl.target, P, int8=wl.weights_int8)
        dft = oracle.Oracle(wl.target.with_layers(wl.draft_layers), DP, int8=wl.weights_int8)

        def one(i):
            out, _, _ = oracle.oracle_generate_speculative(tgt, dft, prompts[i % wl.batch][None], new_per_step,
                                                           wl.lookahead, wl.temperature, seed=1000 + i)
            return out.shape[1] - wl.prompt_len
    for i in range(args.warmup):
        one(i)
    t0 = time.perf_counter()
    toks = 0
    for i in range(args.steps):
        toks += one(args.warmup + i)
    dt = time.perf_counter() - t0
    v = toks / dt
    line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": config_dict(wl, args),
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": ncores, "kind": kind,
                             "sample": f"{args.steps} generate_speculative calls, 1 request x {new_per_step} new tokens each"},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def config_dict(wl, args):
    idx = {"int8": 1, "medium": 2, "tree": 3, "large": 4}.get(wl.name, 1)
    return {"workload": f"{wl.name} (BASELINE configs[{idx}])", "arch": args.arch,
            "model": f"L{wl.target.n_layers} d{wl.target.d_model} H{wl.target.n_heads} F{wl.target.d_ff} V{wl.target.vocab}",
            "draft": f"first {wl.draft_layers} layer(s) + shared head", "batch_per_gpu": wl.batch,
            "global_batch": wl.batch * args.gpus, "prompt_len": wl.prompt_len, "max_new": wl.max_new,
            "lookahead": wl.lookahead, "temperature": wl.temperature, "weights": "int8" if wl.weights_int8 else "f32",
            "act": "bf16" if wl.act_bf16 else "f32", "kv": ["f32", "bf16", "int8"][wl.kv_mode],
            "rng": "philox host uniforms", "tree": list(wl.tree) if wl.tree else None,
            "parallelism": f"request-parallel x{args.gpus}", "l2": "flushed between timed steps (256 MiB write)",
            **({"requests": f"{wl.batch} per GPU: configs[4]'s 256 requests split over 8 GPUs"}
               if wl.name == "large" else {})}


def cpu_baseline_sample(wl):
    """The reference on this host, bounded to ~10-30 s of CPU work."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    kind = "reference" if oracle.reference_available() else "port"
    P = make_params(wl.target, seed=0)
    small = wl.name == "int8"
    nreq = 2 if small else 1
    prompts = make_prompts(nreq, wl.prompt_len, wl.target.vocab, seed=1)
    om = oracle.Oracle(wl.target, P, int8=wl.weights_int8)
    new = 64 if small else 8
    t0 = time.perf_counter()
    toks = 0
    if kind == "reference":
        Pq = [om.param(i).reshape(np.shape(P[i])) for i in range(len(P))]
        tgt = oracle.Reference(wl.target, Pq, requires_grad=False)
        dft = oracle.Reference(wl.target.with_layers(wl.draft_layers), draft_params(wl.target, Pq, wl.draft_layers),
                               requires_grad=False)
        for b in range(nreq):
            toks += len(tgt.generate_speculative(dft, prompts[b], new, wl.lookahead, wl.temperature, 0, 1.0, 7 + b)) - wl.prompt_len
    else:
        dft = oracle.Oracle(wl.target.with_layers(wl.draft_layers), draft_params(wl.target, P, wl.draft_layers),
                            int8=wl.weights_int8)
        out, _, _ = oracle.oracle_generate_speculative(om, dft, prompts, new, wl.lookahead, wl.temperature, seed=7,
                                                       n_threads=1)
        toks = out.size - prompts.size
    dt = time.perf_counter() - t0
    what = "k = 4 chain speculation (the reference has no token trees), " if wl.tree else ""
    return {"value": toks / dt, "unit": UNIT, "cores": os.cpu_count() if kind == "reference" else 1, "kind": kind,
            "sample": f"{what}{nreq} request(s) x {new} new tokens of the same models and prompts, batch 1 each "
                      "(the reference is batch-1)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--arch", default="ref", choices=["ref", "cfg"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="int8", choices=["int8", "medium", "tree", "large"],
                    help="int8 = BASELINE configs[1] (the metric's config, default); medium = configs[2]; "
                         "tree = configs[3]; large = configs[4] at 32 requests per GPU (its 256 over 8 GPUs)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    rank, world, local = dist_env()
    wl = workload(args.workload, ARCH_CFG if args.arch == "cfg" else ARCH_REF)
    large = wl.name == "large"
    if large:
        wl = dataclasses.replace(wl, batch=LARGE_REQUESTS_PER_GPU)
    if args.impl == "reference":
        return reference_arm(args, wl, rank, world)

    import torch
    import torch.distributed as dist

    import specdec_b200 as sd
    from specdec_b200.shard import max_over_ranks, shard

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", init_method="env://", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    t_setup = time.perf_counter()
    P = device_params(wl.target, 0, torch.device("cuda", local)) if large else make_params(wl.target, seed=0)
    eng = sd.Engine(wl.target, draft_layers=wl.draft_layers, weight_dtype=sd.INT8 if wl.weights_int8 else sd.F32,
                    act_dtype=sd.BF16 if wl.act_bf16 else sd.F32, kv_dtype=KV_DTYPE[wl.kv_mode],
                    max_batch=wl.batch, max_lookahead=wl.lookahead, max_prompt_len=wl.prompt_len, device=local,
                    max_tree_nodes=tree_nodes(wl.tree) if wl.tree else 0)
    eng.load_params(sd.TARGET, P)
    del P
    if rank == 0:
        print(f"[bench] weights made and loaded in {time.perf_counter() - t_setup:.1f} s", file=sys.stderr, flush=True)
    B, S = wl.batch, wl.prompt_len
    # request partition: rank r serves requests [r*B, (r+1)*B) of the global set
    prompts = shard(make_prompts(B * world, S, wl.target.vocab, seed=1), B, rank, world)
    n_rounds = wl.max_new + 2
    slots = (len(wl.tree) * max(wl.tree) + 1) if wl.tree else 2 * wl.lookahead + 1
    uni = shard(sd.philox_uniforms(1234, B * world, n_rounds, slots), B, rank, world)

    dev = torch.device("cuda", local)
    d_prompts = torch.from_numpy(prompts.astype(np.int32)).to(dev)
    out_len = S + wl.max_new
    d_out = torch.zeros((B, out_len), dtype=torch.int32, device=dev)
    d_stats = torch.zeros((B, 4), dtype=torch.int64, device=dev)
    stream = torch.cuda.ExternalStream(eng.stream, device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def step():
        if wl.tree:
            eng.generate_tree_device(d_prompts.data_ptr(), B, S, d_out.data_ptr(), d_stats.data_ptr(), wl.max_new,
                                     wl.tree, wl.temperature, seed=1234, uniforms=uni)
        else:
            eng.generate_device(d_prompts.data_ptr(), B, S, d_out.data_ptr(), d_stats.data_ptr(), wl.max_new,
                                wl.lookahead, wl.temperature, seed=1234, uniforms=uni)

    for i in range(args.warmup):
        t0 = time.perf_counter()
        step()
        torch.cuda.synchronize()
        if rank == 0:
            print(f"[bench] warm-up step {i}: {time.perf_counter() - t0:.2f} s", file=sys.stderr, flush=True)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches = 0
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            with torch.cuda.stream(stream):
                flush.fill_(float(i))  # L2 flush, outside the timed events
                starts[i].record(stream)
            step()
            with torch.cuda.stream(stream):
                ends[i].record(stream)
            launches += eng.last_launch_count()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    tot_ms = float(sum(step_ms))
    stats = d_stats.cpu().numpy()
    tokens_out = d_out.cpu().numpy()
    new_tokens = B * wl.max_new  # every request reaches max_new (checked below)
    assert tokens_out.shape == (B, out_len)
    rounds = stats[:, 0].max()
    drafted, accepted = stats[:, 1].sum(), stats[:, 2].sum()

    # e2e through the host-buffer C ABI (pinned host memory, copies inside)
    pin_prompts = torch.from_numpy(prompts.astype(np.int32)).pin_memory()
    pin_uni = torch.from_numpy(uni).pin_memory()
    e2e_ms = []
    # (the large workload's steps take seconds each: one e2e step there)
    for i in range(1 if large else max(3, args.steps // 2)):
        with torch.cuda.stream(stream):
            flush.fill_(float(i))
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
        if wl.tree:
            eng.generate_tree(pin_prompts.numpy(), wl.max_new, wl.tree, wl.temperature, seed=1234,
                              uniforms=pin_uni.numpy())
        else:
            eng.generate_speculative(pin_prompts.numpy(), wl.max_new, wl.lookahead, wl.temperature, seed=1234,
                                     uniforms=pin_uni.numpy())
        with torch.cuda.stream(stream):
            e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms.append(e0.elapsed_time(e1))
    e2e_tot = float(sum(e2e_ms))

    # Autoregressive decoding of the same requests on the same kernels
    # (generate_advanced): the speculative path's speed-up over plain decoding.
    ar_ms = []
    if not wl.tree and not large:
        ar_uni = np.ascontiguousarray(uni[:, : wl.max_new, :1])
        for i in range(args.warmup + 3):
            with torch.cuda.stream(stream):
                flush.fill_(float(i))
                a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a0.record(stream)
            eng.generate_advanced_device(d_prompts.data_ptr(), B, S, d_out.data_ptr(), d_stats.data_ptr(),
                                         wl.max_new, wl.temperature, seed=1234, uniforms=ar_uni)
            with torch.cuda.stream(stream):
                a1.record(stream)
            torch.cuda.synchronize()
            if i >= args.warmup:
                ar_ms.append(a0.elapsed_time(a1))
    ar_tot = float(sum(ar_ms)) if ar_ms else 0.0

    tot_ms, e2e_tot, ar_tot = max_over_ranks([tot_ms, e2e_tot, ar_tot], dist if world > 1 else None, dev)
    ms_per_step = tot_ms / args.steps
    value = new_tokens * world * args.steps / (tot_ms / 1e3)
    e2e_value = new_tokens * world * len(e2e_ms) / (e2e_tot / 1e3)

    hbm, peak_kind = peaks()
    tflops = bf16_peak()
    avg_ctx = S + wl.max_new / 2
    ab = algorithmic_bytes_per_round(wl, wl.weights_int8, avg_ctx)
    round_ms = ms_per_step / max(1, rounds)
    round_achieved = ab["total"] / (round_ms * 1e-3) / 1e9
    clocks = clk.summary()

    # Dominant kernels, timed alone on the library's stream with CUDA events
    # (L2 flushed before every launch) over the verify pass's row count.
    R_verify = B * ((tree_nodes(wl.tree) + 1) if wl.tree else (wl.lookahead + 1))
    m = wl.target
    nk = {"ffn_out": (m.d_model, m.d_ff), "ffn_in": (2 * m.d_ff, m.d_model),
          "qkv": (m.d_model + 2 * m.kv_heads * m.head_dim, m.d_model), "head": (m.vocab, m.d_model)}
    probes = {}
    for name, which, layer in (("ffn_out", sd.LIN_FFN_OUT, 0), ("ffn_in", sd.LIN_FFN_IN, 0),
                               ("qkv", sd.LIN_QKV, 1), ("head", sd.LIN_HEAD, wl.target.n_layers - 1)):
        us, nbytes = eng.time_linear(sd.TARGET, layer, which, R_verify, 20, flush.data_ptr(), flush.numel() * 4)
        flops = 2.0 * R_verify * nk[name][0] * nk[name][1]
        probes[name] = {"us": us, "bytes": nbytes, "GBps": nbytes / (us * 1e-6) / 1e9,
                        "TFLOPs": flops / (us * 1e-6) / 1e12, "flops_per_byte": flops / nbytes}
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": ("int8 weights, bf16 activations" if wl.act_bf16 else "int8")
                if wl.weights_int8 else "f32", "data": "synthetic",
                "config": config_dict(wl, args),
                "e2e": {"value": e2e_value, "unit": UNIT,
                        "h2d_bytes_per_step": int(prompts.size * 4 + uni.nbytes),
                        "d2h_bytes_per_step": int(B * out_len * 4 + B * 4 * 8 + 4)},
                "gpu_launches": int(launches),
                "roofline": {**roofline_entry(probes["ffn_out"], hbm, tflops, wl, R_verify),
                             "launch_us": probes["ffn_out"]["us"], "alg_bytes_per_launch": probes["ffn_out"]["bytes"],
                             "peak_source": peak_kind,
                             "other_kernels": {k: v for k, v in probes.items() if k != "ffn_out"},
                             "round": {"alg_bytes": ab["total"], "achieved": round_achieved,
                                       "frac": round_achieved / hbm, "weight_bytes": ab["weights"],
                                       "kv_bytes": ab["kv"],
                                       "weights_frac": ab["weights"] / (round_ms * 1e-3) / 1e9 / hbm}},
                "spec": {"rounds_per_step": int(rounds), "mean_accepted_per_round": float(accepted) / max(1, stats[:, 0].sum()),
                         "acceptance_rate": float(accepted) / max(1, drafted), "round_us": round_ms * 1e3},
                "clocks": clocks}
        if ar_ms:
            line["ar_decode"] = {"value": new_tokens * world * len(ar_ms) / (ar_tot / 1e3), "unit": UNIT,
                                 "what": "generate_advanced (autoregressive, KV cache) of the same requests, "
                                         "models and uniforms on the same kernels, device-resident"}
        if world == 1 and not args.no_cpu_baseline and not large:
            line["cpu_baseline"] = cpu_baseline_sample(wl)
        if large:
            line["cpu_baseline"] = {"value": None, "unit": UNIT, "cores": os.cpu_count(), "kind": "reference",
                                    "sample": "not sampled: the reference dequantises the 6.6 G int8 weights to "
                                              "fp32 (26 GB) on every Dense call; the int8 workload's line "
                                              "carries the CPU baseline"}
        if wl.tree:
            line["tree"] = {"branching": list(wl.tree), "nodes": tree_nodes(wl.tree),
                            "mean_accepted_per_round": line["spec"]["mean_accepted_per_round"]}
        print(json.dumps(line), flush=True)
    eng.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
