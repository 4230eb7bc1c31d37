"""Generates tests/golden/large_shapes.npz: CPU-oracle outputs for a model with
the layer shapes of the large configuration (d_model
4096, 32 heads x 128, SwiGLU FFN 11008, int8 per-channel weights, bf16
activations and KV cache), cut to 2 target layers and a 1-layer draft with a
4096-token vocabulary so that the oracle finishes in minutes on a CPU.

    make -C oracle oracle && python tests/golden/make_large_shapes.py

The weights are not stored: synth.make_params regenerates them from the seed
(numpy's PCG64 stream is the same on every machine).  What is stored is what
the restatement (oracle/specdec_oracle.cpp) returns for them: a few rows of
the forward logits of a 6-token input (GEMV path on the device) and of a
72-token input (tensor-core GEMM path), and the greedy speculative tokens of
two requests with their decision margins.  tests/test_large_shapes_gpu.py
compares the CUDA path with these on a B200.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "neural-network_b200"))

import oracle  # noqa: E402
from specdec_b200.synth import ModelShape, draft_params, make_params, make_prompts  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "large_shapes.npz")

SHAPE = dict(vocab=4096, d_model=4096, n_heads=32, d_ff=11008, n_layers=2, max_seq_len=128)
DRAFT_LAYERS = 1
SEED = 51
SHORT_S, SHORT_ROWS = 6, (0, 5)
LONG_S, LONG_ROWS = 72, (0, 35, 71)
B, PROMPT, MAX_NEW, K = 2, 16, 20, 4


def main() -> None:
    oracle.build(ref=False)
    shape = ModelShape(**SHAPE)
    P = make_params(shape, seed=SEED, bias_std=0.02, ln_jitter=0.05)
    t = oracle.Oracle(shape, P, int8=True)
    d = oracle.Oracle(shape.with_layers(DRAFT_LAYERS), draft_params(shape, P, DRAFT_LAYERS), int8=True)
    out = {"shape": np.array([SHAPE[k] for k in ("vocab", "d_model", "n_heads", "d_ff", "n_layers", "max_seq_len")]),
           "seed": np.array(SEED)}
    short = make_prompts(1, SHORT_S, shape.vocab, seed=52)[0]
    out["short_tokens"] = short
    out["short_logits"] = t.forward(short, act_bf16=True, kv_mode=1)[list(SHORT_ROWS)]
    long_ = make_prompts(1, LONG_S, shape.vocab, seed=53)[0]
    out["long_tokens"] = long_
    out["long_logits"] = t.forward(long_, act_bf16=True, kv_mode=1)[list(LONG_ROWS)]
    prompts = make_prompts(B, PROMPT, shape.vocab, seed=54)
    tok, stats, mg = oracle.oracle_generate_speculative(t, d, prompts, MAX_NEW, K, 0.0, act_bf16=True, kv_mode=1,
                                                        cache_cap=shape.max_seq_len)
    out["prompts"] = prompts
    out["greedy_tokens"] = tok
    out["greedy_stats"] = stats
    out["greedy_margins"] = mg
    np.savez_compressed(OUT, **out)
    print(OUT, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
