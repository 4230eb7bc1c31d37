"""Shared helpers for the parity tests: build a B200 engine and the CPU
oracle on the same seeded weights and compare their outputs under the
near-tie policy (a token may differ only where the oracle's own decision
margin was below the tolerance; everything after that point in the same
request is then not compared, because the sequences have forked)."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np

import oracle
import specdec_b200 as sd
from specdec_b200.synth import ModelShape, draft_params, make_params, make_prompts

# Decision-margin thresholds below which a token mismatch counts as a near-tie.
GREEDY_REL_GAP = 1e-4      # relative top-2 logit gap
SAMPLED_MARGIN = 2e-5      # |r*q - p| or |cdf - u|
# With bf16 activations every layer output is rounded to 8 significant bits,
# so logits agree to about 1e-2 relative (the bf16 logits tolerance is 2e-2):
# a greedy mismatch is a near-tie below this relative top-2 gap.
BF16_GREEDY_GAP = 2e-2


@dataclass
class Pair:
    shape: ModelShape
    draft_layers: int
    params: list
    dparams: list
    engine: sd.Engine
    target: oracle.Oracle
    draft: oracle.Oracle
    int8: bool
    act_bf16: bool
    kv_mode: int


def make_pair(shape: ModelShape, draft_layers: int, seed: int = 0, int8: bool = False, act_bf16: bool = False,
              kv_mode: int = 0, max_batch: int = 4, max_lookahead: int = 4, max_prompt_len: int = 64,
              bias_std: float = 0.02, ln_jitter: float = 0.05, head_std: Optional[float] = None,
              max_tree_nodes: int = 0, kv_pages: int = 0) -> Pair:
    P = make_params(shape, seed=seed, bias_std=bias_std, ln_jitter=ln_jitter, head_std=head_std)
    DP = draft_params(shape, P, draft_layers)
    eng = sd.Engine(shape, draft_layers=draft_layers, weight_dtype=sd.INT8 if int8 else sd.F32,
                    act_dtype=sd.BF16 if act_bf16 else sd.F32,
                    kv_dtype={0: sd.F32, 1: sd.BF16, 2: sd.INT8}[kv_mode],
                    max_batch=max_batch, max_lookahead=max_lookahead, max_prompt_len=max_prompt_len,
                    max_tree_nodes=max_tree_nodes, kv_pages=kv_pages)
    eng.load_params(sd.TARGET, P)
    t = oracle.Oracle(shape, P, int8=int8)
    d = oracle.Oracle(shape.with_layers(draft_layers), DP, int8=int8)
    return Pair(shape, draft_layers, P, DP, eng, t, d, int8, act_bf16, kv_mode)


def compare_tokens(gpu: np.ndarray, ref: np.ndarray, margins: np.ndarray, prompt_len: int, greedy: bool,
                   tol: Optional[float] = None):
    """Returns (n_exact_requests, n_near_ties).  Raises on a real mismatch."""
    if tol is None:
        tol = GREEDY_REL_GAP if greedy else SAMPLED_MARGIN
    exact, ties = 0, 0
    assert gpu.shape == ref.shape, (gpu.shape, ref.shape)
    for b in range(gpu.shape[0]):
        g, r = gpu[b, prompt_len:], ref[b, prompt_len:]
        assert np.array_equal(gpu[b, :prompt_len], ref[b, :prompt_len])
        diff = np.nonzero(g != r)[0]
        if diff.size == 0:
            exact += 1
            continue
        t = int(diff[0])
        m = float(np.min(margins[b, : t + 1])) if margins is not None else np.inf
        if m >= tol:
            raise AssertionError(
                f"request {b}: token {t} differs (gpu {g[t]} vs oracle {r[t]}) with oracle margin {m:.3g} >= {tol}\n"
                f"gpu    {g[: t + 4].tolist()}\noracle {r[: t + 4].tolist()}")
        ties += 1
    return exact, ties


def run_both(pair: Pair, B: int, S: int, max_new: int, k: int, T: float, seed: int = 42, use_uniforms: bool = False,
             catchup: int = 0, prompt_seed: int = 1, top_k: int = 0, top_p: float = 1.0):
    prompts = make_prompts(B, S, pair.shape.vocab, seed=prompt_seed)
    uni = None
    if use_uniforms:
        uni = sd.philox_uniforms(seed, B, max_new + 2, 2 * k + 1)
    tok_g, st_g = pair.engine.generate_speculative(prompts, max_new, k, T, top_k, top_p, seed, uniforms=uni,
                                                   draft_catchup=catchup)
    tok_o, st_o, mg = oracle.oracle_generate_speculative(
        pair.target, pair.draft, prompts, max_new, k, T, top_k, top_p, seed, uniforms=uni, catchup=catchup,
        act_bf16=pair.act_bf16, kv_mode=pair.kv_mode, cache_cap=pair.shape.max_seq_len)
    return prompts, tok_g, st_g, tok_o, st_o, mg
