"""Generates tests/golden/config_shapes.npz: CPU-oracle outputs at the layer
shapes, batch sizes, lookaheads and temperatures of BASELINE configs[2],
configs[3] and configs[4], with the models cut to 2 target layers (and a
1-layer draft) so that the restatement finishes in minutes on a CPU.

    make -C oracle oracle && python tests/golden/make_config_shapes.py

The weights are not stored: synth.make_params regenerates them from the seeds
(numpy's PCG64 stream is the same on every machine); the prompts and Philox
uniforms are regenerated too.  What is stored is what the restatement
(oracle/specdec_oracle.cpp) returns: tokens, statistics and decision margins.
tests/test_config_shapes_gpu.py compares the CUDA path with them on a B200.

  medium  configs[2]: d_model 768, 12 heads x 64, SwiGLU 3072, vocab 32000,
          int8 weights, bf16 activations and KV cache; 32 requests with
          256-token prompts, k = 6, T = 0.8, Philox uniforms (a 224-row verify
          pass: the tensor-core GEMM with split-K)
  tree    configs[3]: the same model, a 4/3/2/1 token tree (64 nodes) over
          512-token prompts, 8 requests, greedy and T = 1 with uniforms (the
          tensor-core attention walks 5 cache tiles under the ancestor mask)
  large   configs[4]: d_model 4096, 32 heads x 128, SwiGLU 11008 (vocab 4096),
          32 requests, k = 4: a 160-row verify pass (the tensor-core GEMM with
          split-K at K = 11008, the head_dim-128 decode attention), greedy
"""
from __future__ import annotations

import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "neural-network_b200"))

import oracle  # noqa: E402
from specdec_b200.synth import ModelShape, draft_params, make_params, make_prompts, philox_uniforms  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "config_shapes.npz")

MEDIUM = dict(vocab=32000, d_model=768, n_heads=12, d_ff=3072, n_layers=2, max_seq_len=640)
LARGE = dict(vocab=4096, d_model=4096, n_heads=32, d_ff=11008, n_layers=2, max_seq_len=64)

CASES = {
    # name: (shape, seed, B, prompt, max_new, k or tree, temperature, uniforms seed or None)
    "medium": (MEDIUM, 61, 32, 256, 16, 6, 0.8, 611),
    "tree_greedy": (MEDIUM, 62, 8, 512, 12, (4, 3, 2, 1), 0.0, None),
    "tree_sampled": (MEDIUM, 62, 8, 512, 12, (4, 3, 2, 1), 1.0, 621),
    "large": (LARGE, 63, 32, 16, 8, 4, 0.0, None),
}


def models(shape_kw, seed):
    shape = ModelShape(**shape_kw)
    P = make_params(shape, seed=seed, bias_std=0.02, ln_jitter=0.05)
    t = oracle.Oracle(shape, P, int8=True)
    d = oracle.Oracle(shape.with_layers(1), draft_params(shape, P, 1), int8=True)
    return shape, t, d


def case_inputs(name):
    shape_kw, seed, B, S, new, k, T, useed = CASES[name]
    prompts = make_prompts(B, S, shape_kw["vocab"], seed=seed + 1000)
    uni = None
    if useed is not None:
        slots = (len(k) * max(k) + 1) if isinstance(k, tuple) else 2 * k + 1
        uni = philox_uniforms(useed, B, new + 2, slots)
    return prompts, uni


def main() -> None:
    oracle.build(ref=False)
    out = {}
    cache = {}
    for name, (shape_kw, seed, B, S, new, k, T, useed) in CASES.items():
        t0 = time.time()
        key = (tuple(sorted(shape_kw.items())), seed)
        if key not in cache:
            cache[key] = models(shape_kw, seed)
        shape, t, d = cache[key]
        prompts, uni = case_inputs(name)
        if isinstance(k, tuple):
            tok, stats, mg = oracle.oracle_generate_tree(t, d, prompts, new, list(k), T, seed=useed or 0, uniforms=uni,
                                                         act_bf16=True, kv_mode=1, cache_cap=shape.max_seq_len)
        else:
            tok, stats, mg = oracle.oracle_generate_speculative(t, d, prompts, new, k, T, seed=useed or 0,
                                                                uniforms=uni, act_bf16=True, kv_mode=1,
                                                                cache_cap=shape.max_seq_len)
        out[f"{name}_tokens"] = tok
        out[f"{name}_stats"] = stats
        out[f"{name}_margins"] = mg
        print(name, f"{time.time() - t0:.1f} s", stats.sum(axis=0).tolist(), flush=True)
    np.savez_compressed(OUT, **out)
    print(OUT)


if __name__ == "__main__":
    main()
