#!/usr/bin/env python3
"""Benchmark of the B200 speculative-decoding path.

Default workload ("large", the metric's config): target
decoder with 32 layers, d_model 4096, 32 heads x 128, SwiGLU 11008, vocab
32000, int8 per-channel weights, bf16 activations and KV cache; draft = the
target's first 4 layers + shared lm_head; 2048-token uniform-random prompts,
k = 4, temperature 1 with Philox uniforms from the host, 512 new tokens per
request.  BASELINE splits its 256 requests over 8 GPUs; every GPU serves 32 of
them (one GPU's share at 8 GPUs), so the line is weak scaling from 1 GPU.
Weights are seeded synthetic (no checkpoints exist for this path).

One step = one speculative round (k draft steps, one verify pass over the
k+1 rows of every request, acceptance and rollback) of the GPU's 32 requests,
through the round-level session API (specdec_prefill once, untimed; then
specdec_step per step).  `value` is new tokens per second over all GPUs with
everything resident in HBM; `e2e` is the same through the host-buffer C ABI
(each step uploads its rounds' uniforms and downloads the new tokens and
counts inside the timed region).  The line also carries BASELINE configs[1]
("int8": 4 layers, d_model 256, 8 requests, 64-token prompts, 256 new tokens,
one step = one whole generation) under "configs1".

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                  [--workload large|int8|medium|tree]

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

from specdec_b200.synth import (ARCH_CFG, ARCH_REF, device_param_tensors, device_params,  # noqa: E402
                                 draft_params, make_params, make_prompts, workload)

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

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of
# each workload's roofline kernel from an ncu capture of the same launch
# (caches flushed before it, as the live probe does); None until captured.
TRAFFIC_BYTES = {
    "int8": 503808,
    # attn_dec_kernel<8>, verify pass, 32 requests x ~2,060 positions: the
    # one-layer capture of the same launch (1,145.9 MB read + 19.7 MB written)
    "large": 1145909000 + 19673088,
}


def roofline_entry(p, hbm, tflops, wl, rows):
    """The FFN down-projection at the verify row count: HBM-bound below the
    bf16 ridge (peak flops / peak bytes), tensor-bound above it."""
    ridge = tflops * 1e12 / (hbm * 1e9)
    what = "tcgen05 GEMM" if (wl.act_bf16 and rows >= 64) else "linear_kernel GEMV"
    kern = f"{what}, residual epilogue (target FFN down-projection, {rows} verify rows)"
    traffic = TRAFFIC_BYTES.get(wl.name)
    extra = {"kernel": kern}
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
                                          "--format=csv,noheader,nounits", "-lms", "50"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        # nvidia-smi takes a while to start: wait (up to 3 s, before the
        # timed region) for its first sample, so the samples cover the region
        t0 = time.perf_counter()
        while self.proc is not None and time.perf_counter() - t0 < 3.0:
            self.f.flush()
            if os.path.getsize(self.path) > 0 or self.proc.poll() is not None:
                break
            time.sleep(0.02)
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




# ---------------------------------------------------------------------------
# The reference's own CPU implementation (oracle/_ref: the unmodified library)
# on the large workload's models, as a bounded sample.
class _LazyParams:
    """The large models' parameters, made one at a time while the reference
    copies them in (the whole fp32 model is 27 GB): N(0, 0.02) weights and
    embedding, N(0, 4/sqrt(d)) lm_head, zero biases, unit LayerNorm gamma,
    taken from one seeded block of normals.  The sample times the
    reference's work, which does not depend on the values."""

    def __init__(self, shape, n_layers_kept=None):
        from specdec_b200.synth import param_kinds, param_shapes, params_per_layer

        shapes, kinds = param_shapes(shape), param_kinds(shape)
        if n_layers_kept is not None:  # the draft: first layers + the shared head
            per = params_per_layer(shape)
            keep = list(range(1 + per * n_layers_kept)) + [len(shapes) - 2, len(shapes) - 1]
            shapes = [shapes[i] for i in keep]
            kinds = [kinds[i] for i in keep]
        self.shapes, self.kinds, self.d = shapes, kinds, shape.d_model
        self.block = np.random.default_rng(0).standard_normal(1 << 24, dtype=np.float32)

    def __len__(self):
        return len(self.shapes)

    def __iter__(self):
        for shape, kind in zip(self.shapes, self.kinds):
            n = int(np.prod(shape))
            if kind in ("emb", "w", "head_w"):
                std = 4.0 / np.sqrt(self.d) if kind == "head_w" else 0.02
                reps = (n + self.block.size - 1) // self.block.size
                a = np.tile(self.block * np.float32(std), reps)[:n]
            elif kind == "g":
                a = np.ones(n, np.float32)
            else:
                a = np.zeros(n, np.float32)
            yield a


_REF_LARGE = {}
REF_SAMPLE_PROMPT = 32
REF_SAMPLE_NEW = 2


def reference_large_models(wl):
    """The reference TransformerDecoder pair of configs[4] (fp32 Dense weights:
    the reference's QuantizedDense would dequantise all 6.6 G int8 weights
    again on every call)."""
    if "pair" not in _REF_LARGE:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle

        if not oracle.reference_available():
            raise RuntimeError("oracle/_ref/libnnref.so is not built")
        avail = 0
        with open("/proc/meminfo") as f:
            for ln in f:
                if ln.startswith("MemAvailable:"):
                    avail = int(ln.split()[1]) * 1024
        if avail < 48 << 30:
            raise MemoryError(f"the fp32 reference models need ~31 GB of host memory; {avail >> 30} GB available")
        shape = dataclasses.replace(wl.target, max_seq_len=REF_SAMPLE_PROMPT + 4 * REF_SAMPLE_NEW + 16)
        tgt = oracle.Reference(shape, _LazyParams(shape), requires_grad=False)
        dft = oracle.Reference(shape.with_layers(wl.draft_layers), _LazyParams(shape, wl.draft_layers),
                               requires_grad=False)
        _REF_LARGE["pair"] = (tgt, dft)
    return _REF_LARGE["pair"]


def reference_large_call(wl, i):
    """One generate_speculative call of the sample: 1 request, a 32-token
    prompt, 2 new tokens (the first token and one round), k = 4, T = 1."""
    tgt, dft = reference_large_models(wl)
    prompt = make_prompts(1, REF_SAMPLE_PROMPT, wl.target.vocab, seed=100 + i)[0]
    out = tgt.generate_speculative(dft, prompt, REF_SAMPLE_NEW, wl.lookahead, wl.temperature, 0, 1.0, 1000 + i)
    return len(out) - REF_SAMPLE_PROMPT


REF_LARGE_SAMPLE_TEXT = (f"1 request per step: generate_speculative of configs[4]'s target and 4-layer draft (fp32 "
                         f"Dense weights), {REF_SAMPLE_PROMPT}-token prompt, {REF_SAMPLE_NEW} new tokens, k = 4, T = 1; "
                         "the reference is batch-1 and its prefill of a 2048-token prompt alone is ~27 TFLOP")


def reference_arm(args, wl, rank, world):
    """The reference's own CPU implementation on this host's cores, on this
    arm's workload; rank 0 alone runs it (one process; the reference is batch
    1 and uses every host core through its thread pool and OpenBLAS)."""
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("gloo", init_method="env://")
    try:
        if rank == 0:
            _reference_arm_rank0(args, wl)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


def _reference_arm_rank0(args, wl):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # the reference arm times the reference (oracle/_ref) or the CPU restatement

    ncores = os.cpu_count() or 1
    if wl.name == "large":
        kind = "reference"
        t0 = time.perf_counter()
        reference_large_models(wl)
        print(f"[bench] reference models built in {time.perf_counter() - t0:.1f} s", file=sys.stderr, flush=True)
        one = lambda i: reference_large_call(wl, i)  # noqa: E731
        sample = REF_LARGE_SAMPLE_TEXT
    else:
        kind = "reference" if oracle.reference_available() else "port"
        P = make_params(wl.target, seed=0)
        DP = draft_params(wl.target, P, wl.draft_layers)
        new_per_step = 32 if wl.name == "int8" else 8
        prompts = make_prompts(wl.batch, wl.prompt_len, wl.target.vocab, seed=1)
        sample = f"1 request x {new_per_step} new tokens per step (generate_speculative)"
        if kind == "reference":
            # int8 target: the reference multiplies by the dequantised weight q*s
            # (src/nn/quantization.cpp:127-147); inject those values.
            om = oracle.Oracle(wl.target, P, int8=wl.weights_int8)
            Pq = [om.param(i).reshape(np.shape(P[i])) for i in range(len(P))]
            tgt = oracle.Reference(wl.target, Pq, requires_grad=False)
            dft = oracle.Reference(wl.target.with_layers(wl.draft_layers),
                                   draft_params(wl.target, Pq, wl.draft_layers), requires_grad=False)

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
            "impl": "reference", "processes": 1,
            "note": "one host process on rank 0 whatever the GPU count (the reference is batch-1 CPU code)",
            "config": config_dict(wl, args),
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": ncores, "kind": kind, "sample": sample},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def config_dict(wl, args):
    idx = {"int8": 1, "medium": 2, "tree": 3, "large": 4}.get(wl.name, 1)
    step = ("one speculative round of every request (session API)" if wl.name == "large"
            else "one whole generation (generate call)")
    return {"workload": f"{wl.name} (BASELINE configs[{idx}])", "arch": args.arch,
            "model": f"L{wl.target.n_layers} d{wl.target.d_model} H{wl.target.n_heads} F{wl.target.d_ff} V{wl.target.vocab}",
            "draft": f"first {wl.draft_layers} layer(s) + shared head", "batch_per_gpu": wl.batch,
            "global_batch": wl.batch * args.gpus, "prompt_len": wl.prompt_len, "max_new": wl.max_new,
            "lookahead": wl.lookahead, "temperature": wl.temperature, "weights": "int8" if wl.weights_int8 else "f32",
            "act": "bf16" if wl.act_bf16 else "f32", "kv": ["f32", "bf16", "int8"][wl.kv_mode],
            "rng": "philox host uniforms", "tree": list(wl.tree) if wl.tree else None, "step": step,
            "parallelism": f"request-parallel x{args.gpus}",
            "l2": ("inputs larger than L2: 6.6 GB of int8 weights and ~40 GB of KV cache read per step"
                   if wl.name == "large" else "flushed between timed steps (256 MiB write)"),
            **({"requests": f"{wl.batch} per GPU: configs[4]'s 256 requests split over 8 GPUs",
                "kv_pages": f"{kv_pages_needed(wl)} pages of 128 positions per model "
                            f"(prompt + new tokens + one verify block + the draft's catch-up drift)"}
               if wl.name == "large" else {})}


def kv_pages_needed(wl):
    """Pages of the paged KV cache a generation of the workload reserves:
    prompt + new tokens + one verify block, plus the reference catch-up's
    drift of the draft cache (one position per rejected round, at most
    max_new)."""
    return wl.batch * -(-(wl.prompt_len + 2 * wl.max_new + wl.lookahead + 1) // 128)


def cpu_baseline_sample(wl):
    """The reference on this host, bounded to ~10-30 s of CPU work."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    if wl.name == "large":
        reference_large_models(wl)
        t0 = time.perf_counter()
        toks = sum(reference_large_call(wl, i) for i in range(2))
        dt = time.perf_counter() - t0
        return {"value": toks / dt, "unit": UNIT, "cores": os.cpu_count(), "kind": "reference",
                "sample": REF_LARGE_SAMPLE_TEXT.replace("per step", "x 2 calls")}
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


def make_engine(sd, wl, local, large):
    """The engine with seeded synthetic weights.  The large model's weights are
    drawn on the GPU and loaded from there (quantised and transposed on the
    device): every rank of a multi-GPU run would otherwise hold a 27 GB fp32
    copy in host memory."""
    import torch

    eng = sd.Engine(wl.target, draft_layers=wl.draft_layers, weight_dtype=sd.INT8 if wl.weights_int8 else sd.F32,
                    act_dtype=sd.BF16 if wl.act_bf16 else sd.F32, kv_dtype=KV_DTYPE[wl.kv_mode],
                    max_batch=wl.batch, max_lookahead=wl.lookahead, max_prompt_len=wl.prompt_len, device=local,
                    max_tree_nodes=tree_nodes(wl.tree) if wl.tree else 0,
                    kv_pages=kv_pages_needed(wl) if large else 0)
    if large:
        P = device_param_tensors(wl.target, 0, torch.device("cuda", local))
        eng.load_params_device(sd.TARGET, P)
        del P
        torch.cuda.empty_cache()
    else:
        eng.load_params(sd.TARGET, make_params(wl.target, seed=0))
    return eng


def linear_probes(sd, eng, wl, R_verify, flush):
    """The verify pass's linear layers, timed alone on the library's stream
    with CUDA events (L2 flushed before every launch)."""
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
    return probes


def run_generate_bench(args, wl, rank, world, local, dist):
    """Workloads int8 / medium / tree: one step = one whole generation."""
    import torch

    import specdec_b200 as sd
    from specdec_b200.shard import max_over_ranks, shard

    t_setup = time.perf_counter()
    eng = make_engine(sd, wl, local, False)
    if rank == 0:
        print(f"[bench] {wl.name}: weights made and loaded in {time.perf_counter() - t_setup:.1f} s",
              file=sys.stderr, flush=True)
    B, S = wl.batch, wl.prompt_len
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
        step()
        torch.cuda.synchronize()
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
    tot_ms = float(sum(s.elapsed_time(e) for s, e in zip(starts, ends)))
    stats = d_stats.cpu().numpy()
    tokens_out = d_out.cpu().numpy()
    # every request reaches max_new new tokens, within the vocabulary
    n_new = stats[:, 0]
    assert tokens_out.shape == (B, out_len)
    assert np.array_equal(tokens_out[:, :S], prompts.astype(np.int32)), "prompts were not kept"
    assert ((tokens_out[:, S:] >= 0) & (tokens_out[:, S:] < wl.target.vocab)).all(), "token out of range"
    new_tokens = B * wl.max_new
    checks = {"requests_complete": True, "tokens_in_vocab": True}
    if not wl.tree and rank == 0 and wl.name == "int8":
        # request 0 against the CPU restatement on the same weights and uniforms
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle

        P = make_params(wl.target, seed=0)
        om = oracle.Oracle(wl.target, P, int8=wl.weights_int8)
        dm = oracle.Oracle(wl.target.with_layers(wl.draft_layers), draft_params(wl.target, P, wl.draft_layers),
                           int8=wl.weights_int8)
        ref, _, mg = oracle.oracle_generate_speculative(om, dm, prompts[:1], wl.max_new, wl.lookahead,
                                                        wl.temperature, seed=1234, uniforms=uni[:1],
                                                        cache_cap=wl.target.max_seq_len)
        diff = np.nonzero(ref[0] != tokens_out[0])[0]
        first = int(diff[0]) - S if diff.size else -1
        tie = bool(diff.size == 0 or float(mg[0, : first + 1].min()) < 2e-5)
        checks["request0_equals_oracle"] = bool(diff.size == 0)
        checks["request0_first_difference"] = first
        assert tie, f"request 0 differs from the oracle at new token {first}"
    rounds = stats[:, 0].max()
    drafted, accepted = stats[:, 1].sum(), stats[:, 2].sum()
    del n_new

    # e2e through the host-buffer C ABI (pinned host memory, copies inside)
    pin_prompts = torch.from_numpy(prompts.astype(np.int32)).pin_memory()
    pin_uni = torch.from_numpy(uni).pin_memory()
    e2e_ms = []
    for i in range(max(3, args.steps // 2)):
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
    if not wl.tree:
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
    R_verify = B * ((tree_nodes(wl.tree) + 1) if wl.tree else (wl.lookahead + 1))
    probes = linear_probes(sd, eng, wl, R_verify, flush)
    eng.close()
    if rank != 0:
        return None
    line = {"metric": METRIC, "value": value, "unit": UNIT, "value_per_gpu": value / world, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": ("int8 weights, bf16 activations" if wl.act_bf16 else "int8") if wl.weights_int8 else "f32",
            "data": "synthetic", "config": config_dict(wl, args),
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(prompts.size * 4 + uni.nbytes),
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
            "checks": checks, "clocks": clocks}
    if ar_ms:
        line["ar_decode"] = {"value": new_tokens * world * len(ar_ms) / (ar_tot / 1e3), "unit": UNIT,
                             "what": "generate_advanced (autoregressive, KV cache) of the same requests, "
                                     "models and uniforms on the same kernels, device-resident"}
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_sample(wl)
    if wl.tree:
        line["tree"] = {"branching": list(wl.tree), "nodes": tree_nodes(wl.tree),
                        "mean_accepted_per_round": line["spec"]["mean_accepted_per_round"]}
    return line


def run_session_bench(args, wl, rank, world, local, dist):
    """The large workload: prefill once (untimed), one step = one round."""
    import torch

    import specdec_b200 as sd
    from specdec_b200.shard import max_over_ranks, shard, sum_over_ranks

    t_setup = time.perf_counter()
    eng = make_engine(sd, wl, local, True)
    if rank == 0:
        print(f"[bench] {wl.name}: weights made and loaded in {time.perf_counter() - t_setup:.1f} s",
              file=sys.stderr, flush=True)
    B, S, k, T = wl.batch, wl.prompt_len, wl.lookahead, wl.temperature
    R = max(1, args.rounds_per_step)
    prompts = shard(make_prompts(B * world, S, wl.target.vocab, seed=1), B, rank, world)
    slots = 2 * k + 1
    uni = shard(sd.philox_uniforms(1234, B * world, wl.max_new + 2, slots), B, rank, world)
    n_e2e = 0 if args.profile else max(3, args.steps // 2)
    budget = wl.max_new - 2  # rounds a request can take after its first token
    if R * (args.warmup + args.steps + n_e2e) > budget:
        raise SystemExit(f"{R * (args.warmup + args.steps + n_e2e)} rounds exceed the session's {budget}: "
                         "fewer steps or rounds per step")
    dev = torch.device("cuda", local)
    d_prompts = torch.from_numpy(prompts.astype(np.int32)).to(dev)
    cap = R * (k + 1)
    d_tok = torch.zeros((args.steps + args.warmup, B, cap), dtype=torch.int32, device=dev)
    d_cnt = torch.zeros((args.steps + args.warmup, B), dtype=torch.int32, device=dev)
    stream = torch.cuda.ExternalStream(eng.stream, device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    t0 = time.perf_counter()
    eng.prefill_device(d_prompts.data_ptr(), B, S, wl.max_new, k, T, seed=1234, uniforms=uni)
    torch.cuda.synchronize()
    if rank == 0:
        print(f"[bench] prefill of {B} x {S} tokens: {time.perf_counter() - t0:.2f} s", file=sys.stderr, flush=True)

    def step(i):
        eng.step_device(R, d_tok[i].data_ptr(), d_cnt[i].data_ptr(), cap)

    for i in range(args.warmup):
        step(i)
        torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches = 0
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            with torch.cuda.stream(stream):
                starts[i].record(stream)
            step(args.warmup + i)
            with torch.cuda.stream(stream):
                ends[i].record(stream)
            launches += eng.last_launch_count()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    tot_ms = float(sum(step_ms))
    cnt = d_cnt.cpu().numpy()
    tok = d_tok.cpu().numpy()
    timed_tokens = int(cnt[args.warmup:].sum())
    # every request emits at least one token per round, within the vocabulary
    assert (cnt >= R).all(), "a request emitted no token in a round"
    for i in range(cnt.shape[0]):
        for b in range(B):
            t = tok[i, b, : min(cnt[i, b], cap)]
            assert ((t >= 0) & (t < wl.target.vocab)).all(), "token out of range"

    # e2e: the host-buffer step (uploads its rounds' uniforms, downloads the
    # tokens and counts) from pinned host memory
    e2e_ms, e2e_tokens = [], 0
    r0 = 1 + R * (args.warmup + args.steps)
    pin_uni = torch.from_numpy(np.ascontiguousarray(uni)).pin_memory().numpy()
    for i in range(n_e2e):
        u = np.ascontiguousarray(pin_uni[:, r0 + R * i: r0 + R * (i + 1)])
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            e0.record(stream)
        _, c = eng.step(R, uniforms=u)
        with torch.cuda.stream(stream):
            e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms.append(e0.elapsed_time(e1))
        e2e_tokens += int(c.sum())
    e2e_tot = float(sum(e2e_ms))

    # the session's sequences: prompts kept, the step outputs are its new tokens
    full, stats = eng.session_tokens()
    checks = {"tokens_per_round_ge_1": True, "tokens_in_vocab": True}
    emitted = 1 + cnt.sum(axis=0)
    assert np.array_equal(full[:, :S], prompts), "prompts were not kept"
    for b in range(B):
        seq = [int(full[b, S])] + [int(x) for i in range(cnt.shape[0]) for x in tok[i, b, : cnt[i, b]]]
        assert seq == full[b, S: S + int(emitted[b])].tolist(), "step outputs differ from the session's tokens"
    checks["step_outputs_equal_session_tokens"] = True

    # live kernel timings over the session's caches (L2 flushed before each):
    # the verify pass's attention (the dominant kernel) and linear layers
    hbm, peak_kind = peaks()
    tflops = bf16_peak()
    att_us, att_bytes = (eng.time_attention(sd.TARGET, 0, k + 1, 10, flush.data_ptr(), flush.numel() * 4)
                         if not args.profile else (1.0, 0.0))
    R_verify = B * (k + 1)
    probes = linear_probes(sd, eng, wl, R_verify, flush) if not args.profile else {}
    clocks = clk.summary()
    eng.close()

    tot_ms, e2e_tot, att_us = max_over_ranks([tot_ms, e2e_tot, att_us], dist if world > 1 else None, dev)
    timed_tokens, e2e_tokens = sum_over_ranks([timed_tokens, e2e_tokens], dist if world > 1 else None, dev)
    if rank != 0:
        return None
    ms_per_step = tot_ms / args.steps
    value = timed_tokens / (tot_ms / 1e3)
    e2e_value = e2e_tokens / (e2e_tot / 1e3) if e2e_ms else None
    rounds = args.steps * R
    # algorithmic bytes of a round at the timed rounds' average context
    avg_ctx = S + 1 + (args.warmup + args.steps / 2) * R * (1 + float(stats[:, 2].sum()) / max(1, stats[:, 0].sum()))
    ab = algorithmic_bytes_per_round(wl, wl.weights_int8, avg_ctx)
    round_ms = ms_per_step / R
    round_achieved = ab["total"] / (round_ms * 1e-3) / 1e9
    att_gbps = att_bytes / (att_us * 1e-6) / 1e9
    line = {"metric": METRIC, "value": value, "unit": UNIT, "value_per_gpu": value / world, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 weights, bf16 activations and KV",
            "data": "synthetic", "config": {**config_dict(wl, args), "rounds_per_step": R},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(B * R * slots * 4),
                    "d2h_bytes_per_step": int(B * cap * 4 + B * 4 + 4)},
            "gpu_launches": int(launches),
            "roofline": {"bound": "hbm", "achieved": att_gbps, "peak": hbm, "unit": "GB/s", "frac": att_gbps / hbm,
                         "traffic": TRAFFIC_BYTES.get("large"),
                         "kernel": f"attn_dec_kernel (tcgen05 decode attention, head_dim 128), verify pass of "
                                   f"layer 0: {B} requests x {k + 1} rows over ~{int(avg_ctx)} cached positions",
                         "launch_us": att_us, "alg_bytes_per_launch": att_bytes, "peak_source": peak_kind,
                         "other_kernels": probes,
                         "round": {"alg_bytes": ab["total"], "achieved": round_achieved,
                                   "frac": round_achieved / hbm, "weight_bytes": ab["weights"],
                                   "kv_bytes": ab["kv"], "avg_ctx": avg_ctx,
                                   "weights_frac": ab["weights"] / (round_ms * 1e-3) / 1e9 / hbm}},
            "spec": {"rounds_per_step": R, "mean_accepted_per_round": float(stats[:, 2].sum()) / max(1, stats[:, 0].sum()),
                     "acceptance_rate": float(stats[:, 2].sum()) / max(1, stats[:, 1].sum()),
                     "round_us": round_ms * 1e3, "timed_rounds": rounds},
            "checks": checks, "clocks": clocks}
    if world == 1 and not args.no_cpu_baseline and not args.profile:
        try:
            line["cpu_baseline"] = cpu_baseline_sample(wl)
        except (RuntimeError, OSError, MemoryError) as e:
            line["cpu_baseline"] = {"value": None, "unit": UNIT, "cores": os.cpu_count(), "kind": "reference",
                                    "sample": f"not sampled: {e}"}
    return line


def run_tp_bench(args, wl, rank, world, local, dist):
    """BASELINE configs[4]'s tensor-parallel variant: 16 requests served by all
    `world` GPUs together (specdec_create_tp: heads and FFN columns split, an
    NCCL all-reduce after the attention output and FFN down projections).
    Rounds through the session API; every rank returns the same tokens.  The
    all-reduce share is the time of the round's all-reduces (the same sizes,
    timed with torch's NCCL on this group) over the round's time."""
    import hashlib

    import torch

    import specdec_b200 as sd
    from specdec_b200.shard import max_over_ranks

    B, S, k, T = 16, wl.prompt_len, wl.lookahead, wl.temperature
    dev = torch.device("cuda", local)
    obj = [sd.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    eng = sd.Engine(wl.target, draft_layers=wl.draft_layers, weight_dtype=sd.INT8, act_dtype=sd.BF16,
                    kv_dtype=sd.BF16, max_batch=B, max_lookahead=k, max_prompt_len=S, device=local,
                    tp_rank=rank, tp_world=world, tp_id=obj[0],
                    kv_pages=B * -(-(S + 2 * wl.max_new + k + 1) // 128))
    P = device_param_tensors(wl.target, 0, dev)
    eng.load_params_device(sd.TARGET, P)
    del P
    torch.cuda.empty_cache()
    prompts = make_prompts(B, S, wl.target.vocab, seed=2)
    uni = sd.philox_uniforms(4321, B, wl.max_new + 2, 2 * k + 1)
    d_prompts = torch.from_numpy(prompts.astype(np.int32)).to(dev)
    eng.prefill_device(d_prompts.data_ptr(), B, S, wl.max_new, k, T, seed=4321, uniforms=uni)
    torch.cuda.synchronize()
    n_w, n_t = 3, 10
    cap = k + 1
    d_tok = torch.zeros((n_w + n_t, B, cap), dtype=torch.int32, device=dev)
    d_cnt = torch.zeros((n_w + n_t, B), dtype=torch.int32, device=dev)
    stream = torch.cuda.ExternalStream(eng.stream, device=dev)
    for i in range(n_w):
        eng.step_device(1, d_tok[i].data_ptr(), d_cnt[i].data_ptr(), cap)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
    for i in range(n_w, n_w + n_t):
        eng.step_device(1, d_tok[i].data_ptr(), d_cnt[i].data_ptr(), cap)
    with torch.cuda.stream(stream):
        e1.record(stream)
    torch.cuda.synchronize()
    tot_ms = e0.elapsed_time(e1)
    tokens = int(d_cnt[n_w:].sum().item())
    full, _ = eng.session_tokens()
    eng.close()
    digest = hashlib.sha256(np.ascontiguousarray(full).tobytes()).hexdigest()
    digests = [None] * world
    dist.all_gather_object(digests, digest)
    # the round's all-reduces: per layer two of [rows][d_model] bf16 -- the
    # verify pass (B (k + 1) rows, L target layers), draft step 0 (2B rows)
    # and steps 1 .. k-1 (B rows) over the draft's layers
    d = wl.target.d_model
    sizes = ([B * (k + 1)] * (2 * wl.target.n_layers) + [2 * B] * (2 * wl.draft_layers) +
             [B] * (2 * wl.draft_layers * (k - 1)))
    ar_ms = 0.0
    for rows in sorted(set(sizes)):
        x = torch.zeros((rows, d), dtype=torch.bfloat16, device=dev)
        for _ in range(3):
            dist.all_reduce(x)
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a0.record()
        for _ in range(20):
            dist.all_reduce(x)
        a1.record()
        torch.cuda.synchronize()
        ar_ms += a0.elapsed_time(a1) / 20 * sizes.count(rows)
    tot_ms, ar_ms = max_over_ranks([tot_ms, ar_ms], dist, dev)
    if rank != 0:
        return None
    round_ms = tot_ms / n_t
    return {"world": world, "batch": B, "value": tokens / (tot_ms / 1e3), "unit": UNIT, "rounds_timed": n_t,
            "ms_per_round": round_ms, "allreduce_ms_per_round": ar_ms, "allreduce_share": ar_ms / round_ms,
            "allreduces_per_round": len(sizes), "ranks_agree": len(set(digests)) == 1,
            "what": "16 requests on all GPUs together (heads and FFN columns split, NCCL all-reduce after the "
                    "attention output and FFN down projections); all-reduce time = torch's NCCL on the same "
                    "sizes, timed apart"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--arch", default="ref", choices=["ref", "cfg"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="large", choices=["large", "int8", "medium", "tree"],
                    help="large = BASELINE configs[4], the metric's config (default; 32 requests per GPU, one "
                         "step = one round); int8 = configs[1]; medium = configs[2]; tree = configs[3]")
    ap.add_argument("--rounds-per-step", type=int, default=1, help="large workload: speculative rounds per step")
    ap.add_argument("--layers", type=int, default=0,
                    help="target layers (0: the workload's); a cut of the model for profiler captures")
    ap.add_argument("--batch", type=int, default=0,
                    help="requests per GPU (0: the workload's); a smaller case for profiler captures")
    ap.add_argument("--skip-configs1", action="store_true", help="large workload: no configs[1] sub-line")
    ap.add_argument("--no-tp", action="store_true", help="large workload on N > 1 GPUs: no tensor-parallel line")
    ap.add_argument("--profile", action="store_true",
                    help="timed steps only (no e2e, probes, CPU baseline or configs[1]): for profiler launch lists")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    rank, world, local = dist_env()
    wl = workload(args.workload, ARCH_CFG if args.arch == "cfg" else ARCH_REF)
    large = wl.name == "large"
    if large:
        wl = dataclasses.replace(wl, batch=LARGE_REQUESTS_PER_GPU)
    if args.batch:
        wl = dataclasses.replace(wl, batch=args.batch)
    if args.layers:
        wl = dataclasses.replace(wl, target=wl.target.with_layers(args.layers),
                                 draft_layers=min(wl.draft_layers, args.layers))
    if args.impl == "reference":
        return reference_arm(args, wl, rank, world)

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    if world > 1:
        # the tensor-parallel variant's NCCL traffic stays off NVLink
        # multicast (NVLS), as its tests run it
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        from datetime import timedelta
        dist.init_process_group("nccl", init_method="env://", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    try:
        if large:
            line = run_session_bench(args, wl, rank, world, local, dist)
            if world > 1 and not args.profile and not args.no_tp:
                torch.cuda.empty_cache()
                try:
                    tp = run_tp_bench(args, wl, rank, world, local, dist)
                except Exception as e:  # the same on every rank (shapes, memory): the main line stands
                    tp = {"world": world, "error": f"{type(e).__name__}: {e}"[:300]}
                torch.cuda.empty_cache()
                if line is not None:
                    line["tp"] = tp
            if not args.skip_configs1 and not args.profile:
                torch.cuda.empty_cache()
                sub_args = argparse.Namespace(**{**vars(args), "steps": 10, "warmup": 3})
                sub = run_generate_bench(sub_args, workload("int8"), rank, world, local, dist)
                if line is not None and sub is not None:
                    line["configs1"] = {k: sub[k] for k in ("value", "value_per_gpu", "ms_per_step", "e2e", "config",
                                                            "spec", "checks", "gpu_launches") if k in sub}
                    line["configs1"]["round_frac"] = sub["roofline"]["round"]["frac"]
                    if "cpu_baseline" in sub:
                        line["configs1"]["cpu_baseline"] = sub["cpu_baseline"]
        else:
            line = run_generate_bench(args, wl, rank, world, local, dist)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
