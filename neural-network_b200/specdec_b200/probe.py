"""One forward pass, or one speculative generation, of a seeded synthetic model
at a chosen size, for profilers:

    PYTHONPATH=neural-network_b200 python -m specdec_b200.probe --rows 4160
    PYTHONPATH=neural-network_b200 python -m specdec_b200.probe --d-model 4096 --heads 32 --ffn 11008 \\
        --layers 2 --generate 16 --batch 32 --rows 2048 --gpu-weights

Without --generate it runs specdec_forward_logits twice on `rows` uniform-random
tokens of one request (int8 weights, bf16 activations and KV cache by
default).  Every layer of the second call launches the same kernels as the
first, so a profiler that skips the first call's launches captures warm
tensor-core GEMMs (tcgen05) and tensor-core attention at that row count after
a few dozen launches.  The default shape is the medium configuration's layer
(d_model 768, 12 heads x 64, SwiGLU 3072, vocab 32000) cut to 2 layers; 4160
rows is a token-tree verify pass (64 requests x 65 rows).

With --generate N it runs one speculative generation instead: `batch`
requests with `rows`-token prompts, N new tokens, k = --lookahead, a draft of
the target's first --draft-layers layers, temperature 1 with Philox uniforms.
With SPECDEC_NO_GRAPH=1 the library launches the round's kernels directly, so
a profiler sees each of them (the d_model 4096 / 32 x 128 / 11008 shape above
gives the large configuration's per-layer launches).  --gpu-weights draws the
weights with torch on the GPU (synth.device_params), which takes seconds where
numpy takes minutes for multi-GB models; timings do not depend on the values.
"""
from __future__ import annotations

import argparse
import time

from . import BF16, F32, INT8, TARGET, Engine, philox_uniforms
from .synth import ModelShape, device_params, make_params, make_prompts


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--rows", type=int, default=4160, help="forward rows, or the prompt length with --generate")
    ap.add_argument("--d-model", type=int, default=768)
    ap.add_argument("--heads", type=int, default=12)
    ap.add_argument("--ffn", type=int, default=3072)
    ap.add_argument("--vocab", type=int, default=32000)
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--fp32", action="store_true", help="fp32 weights, activations and KV cache")
    ap.add_argument("--generate", type=int, default=0, help="new tokens of one speculative generation")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--lookahead", type=int, default=4)
    ap.add_argument("--draft-layers", type=int, default=1)
    ap.add_argument("--gpu-weights", action="store_true", help="draw the weights with torch on the GPU")
    args = ap.parse_args()
    gen = args.generate > 0
    max_seq = args.rows + (2 * args.generate + 8 if gen else 0)
    shape = ModelShape(vocab=args.vocab, d_model=args.d_model, n_heads=args.heads, d_ff=args.ffn,
                       n_layers=args.layers, max_seq_len=max_seq)
    lo = args.fp32
    t0 = time.perf_counter()
    eng = Engine(shape, draft_layers=args.draft_layers, weight_dtype=F32 if lo else INT8,
                 act_dtype=F32 if lo else BF16, kv_dtype=F32 if lo else BF16, max_batch=args.batch,
                 max_lookahead=args.lookahead, max_prompt_len=args.rows)
    try:
        if args.gpu_weights:
            import torch

            P = device_params(shape, 0, torch.device("cuda", 0))
        else:
            P = make_params(shape, seed=0)
        eng.load_params(TARGET, P)
        del P
        print(f"weights made and loaded in {time.perf_counter() - t0:.1f} s", flush=True)
        if gen:
            prompts = make_prompts(args.batch, args.rows, shape.vocab, seed=1)
            uni = philox_uniforms(1234, args.batch, args.generate + 2, 2 * args.lookahead + 1)
            t0 = time.perf_counter()
            _, stats = eng.generate_speculative(prompts, args.generate, args.lookahead, 1.0, seed=1234, uniforms=uni)
            print(f"generate: {args.batch} x {args.generate} new tokens in {(time.perf_counter() - t0) * 1e3:.1f} ms "
                  f"(host wall clock), {int(stats[:, 0].max())} rounds", flush=True)
            return
        toks = make_prompts(1, args.rows, shape.vocab, seed=1)[0]
        for i in range(2):
            t0 = time.perf_counter()
            eng.forward_logits(TARGET, toks)
            print(f"forward {i}: {args.rows} rows in {(time.perf_counter() - t0) * 1e3:.2f} ms "
                  f"(host wall clock, logits copy included)", flush=True)
    finally:
        eng.close()


if __name__ == "__main__":
    main()
