"""Generates tests/golden/reference_cases.npz from the UNMODIFIED reference.

Run in a container that has the reference tree (its library is compiled from
its own sources by oracle/Makefile into oracle/_ref/libnnref.so):

    make -C oracle ref && python tests/golden/make_golden.py

Every case injects seeded weights (neural-network_b200/specdec_b200/synth.py)
into reference TransformerDecoder objects and records what the reference
returns: forward logits, generate_advanced and generate_speculative tokens in
greedy, sampled (std::mt19937), top-k/top-p and int8-KV modes, and the NETW
v1 weight files the reference writes for two of the targets.  (Logits depend
on OpenBLAS's thread count at the 1e-7 level; the tests allow 1e-5.)  The shapes
include the reference's own test models (tests/nn/transformer_test.cpp:
vocab 8/6, d_model 8, 2 heads, FFN 16, 2 target layers, 1 draft layer) and a
config-1-shaped model cut down to two layers.  These fixtures pin the CPU
restatement (oracle/specdec_oracle.cpp) on machines without the reference.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "neural-network_b200"))

from oracle import Reference, build, ref_quantize_int8, ref_rope  # noqa: E402
from specdec_b200.synth import ModelShape, draft_params, make_params, make_prompts  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_cases.npz")

# (name, shape, draft layers, weight seed, prompt len, bias/ln jitter)
MODELS = [
    ("tiny8", ModelShape(vocab=8, d_model=8, n_heads=2, d_ff=16, n_layers=2, max_seq_len=64), 1, 11, 3, 0.05),
    ("tiny6", ModelShape(vocab=6, d_model=8, n_heads=2, d_ff=16, n_layers=2, max_seq_len=64), 1, 12, 3, 0.05),
    ("small", ModelShape(vocab=97, d_model=32, n_heads=4, d_ff=64, n_layers=2, max_seq_len=160), 1, 13, 9, 0.02),
    ("cfg1cut", ModelShape(vocab=2048, d_model=256, n_heads=4, d_ff=1024, n_layers=2, max_seq_len=96), 1, 0, 6, 0.0),
]

# targets whose NETW v1 weight file (Layer::save_weights) is kept as a fixture
NETW_MODELS = ("tiny8", "small")

# (tag, max_new, lookahead, T, top_k, top_p, seed, quantized_cache)
SPEC_CASES = [
    ("greedy", 12, 3, 0.0, 0, 1.0, 42, False),
    ("greedy_k1", 8, 1, 0.0, 0, 1.0, 42, False),
    ("t1_s1", 16, 3, 1.0, 0, 1.0, 1, False),
    ("t1_s7", 16, 4, 1.0, 0, 1.0, 7, False),
    ("t07_s3", 16, 2, 0.7, 0, 1.0, 3, False),
    ("topk_topp", 12, 3, 1.0, 4, 0.9, 42, False),
    ("qcache_greedy", 10, 2, 0.0, 0, 1.0, 42, True),
    ("qcache_t1", 10, 2, 1.0, 0, 1.0, 5, True),
]


def main() -> None:
    build(ref=True)
    out = {}
    for name, shape, dl, wseed, plen, jit in MODELS:
        P = make_params(shape, seed=wseed, bias_std=jit, ln_jitter=jit)
        DP = draft_params(shape, P, dl)
        dshape = shape.with_layers(dl)
        tgt = Reference(shape, P, requires_grad=False)
        dft = Reference(dshape, DP, requires_grad=False)
        prompt = make_prompts(1, plen, shape.vocab, seed=wseed + 100)[0]
        out[f"{name}/prompt"] = prompt
        out[f"{name}/logits_target"] = tgt.forward(prompt)
        out[f"{name}/logits_draft"] = dft.forward(prompt)
        # the constructor-default (grad-requiring) model takes the unfused path
        out[f"{name}/logits_target_unfused"] = Reference(shape, P, requires_grad=True).forward(prompt)
        n_case = 0
        for tag, mn, k, T, tk, tp, seed, qc in SPEC_CASES:
            if shape.vocab > 200 and tag not in ("greedy", "t1_s1"):
                continue
            out[f"{name}/spec/{tag}"] = tgt.generate_speculative(dft, prompt, mn, k, T, tk, tp, seed, qc)
            out[f"{name}/spec/{tag}/args"] = np.array([mn, k, T, tk, tp, seed, int(qc)], np.float64)
            n_case += 1
        out[f"{name}/ar_greedy"] = tgt.generate_advanced(prompt, 12, 0.0, 0, 1.0, 42, True)
        out[f"{name}/ar_greedy_nocache"] = tgt.generate_advanced(prompt, 12, 0.0, 0, 1.0, 42, False)
        out[f"{name}/ar_t09"] = tgt.generate_advanced(prompt, 12, 0.9, 5, 0.8, 7, True)
        if name in NETW_MODELS:
            # the reference's own weight file of this target (Layer::save_weights)
            tgt.save_weights(os.path.join(os.path.dirname(OUT), f"{name}_target.netw"))
        print(f"{name}: {n_case} speculative cases")
    # known answers of the reference's own unit tests
    x = np.array([1, 2, 3, 4, 5, 6, 7, 8], np.float32).reshape(1, 1, 2, 4)
    out["rope/in"] = x
    out["rope/out"] = ref_rope(x, 0)
    w = np.array([[-1.27, 0.5], [12.7, -6.35]], np.float32)
    s, q, dq = ref_quantize_int8(w)
    out["int8/w"], out["int8/scales"], out["int8/q"], out["int8/dequant"] = w, s, q, dq
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes)")


if __name__ == "__main__":
    main()
