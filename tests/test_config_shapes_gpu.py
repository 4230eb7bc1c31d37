"""The CUDA path at the shapes, batch sizes, lookaheads and temperatures of
BASELINE configs[2] (medium), configs[3] (token tree) and configs[4] (large),
with the models cut to 2 target layers and a 1-layer draft, against the CPU
oracle's outputs for the same seeded weights, prompts and Philox uniforms
(tests/golden/config_shapes.npz, made by tests/golden/make_config_shapes.py).

What the cut keeps: the medium case's 224-row verify pass (32 requests x
(6 + 1)) runs the tensor-core GEMM with split-K and its 32-request draft
steps the wide-layer GEMM; the tree cases run tensor-core attention over
5 cache tiles of a 512-token prompt under the ancestor mask; the large case's
160-row verify runs split-K at K = 11008 and the head_dim-128 decode
attention.  Tolerances are the bf16 ones of the parity contract: tokens exact
up to the first near-tie of the oracle's decision margins."""
import importlib.util
import os

import numpy as np
import pytest

from helpers import BF16_GREEDY_GAP, compare_tokens

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURE = os.path.join(HERE, "golden", "config_shapes.npz")
# sampled decisions under bf16 activations: a mismatch counts as a near-tie
# below this margin (|r q - p| or |cdf - u|)
BF16_SAMPLED_MARGIN = 2e-3


def _gen():
    spec = importlib.util.spec_from_file_location("make_config_shapes",
                                                  os.path.join(HERE, "golden", "make_config_shapes.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_fixture_has_every_case():
    gen = _gen()
    g = np.load(FIXTURE)
    for name, (shape, seed, B, S, new, k, T, useed) in gen.CASES.items():
        assert g[f"{name}_tokens"].shape == (B, S + new)
        prompts, _ = gen.case_inputs(name)
        assert np.array_equal(g[f"{name}_tokens"][:, :S], prompts)


_ENGINES = {}


def _engine(gen, name):
    import specdec_b200 as sd
    from specdec_b200.synth import ModelShape, make_params

    shape_kw, seed, B, S, new, k, T, useed = gen.CASES[name]
    key = (tuple(sorted(shape_kw.items())), seed)
    if key not in _ENGINES:
        for e in _ENGINES.values():
            e.close()
        _ENGINES.clear()
        shape = ModelShape(**shape_kw)
        eng = sd.Engine(shape, draft_layers=1, weight_dtype=sd.INT8, act_dtype=sd.BF16, kv_dtype=sd.BF16,
                        max_batch=32, max_lookahead=6, max_prompt_len=512, max_tree_nodes=64)
        eng.load_params(sd.TARGET, make_params(shape, seed=seed, bias_std=0.02, ln_jitter=0.05))
        _ENGINES[key] = eng
    return _ENGINES[key]


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["medium", "tree_greedy", "tree_sampled", "large"])
def test_config_shapes_match_oracle(gpu_lib, name):
    gen = _gen()
    g = np.load(FIXTURE)
    shape_kw, seed, B, S, new, k, T, useed = gen.CASES[name]
    prompts, uni = gen.case_inputs(name)
    eng = _engine(gen, name)
    if isinstance(k, tuple):
        tok, stats = eng.generate_tree(prompts, new, list(k), T, seed=useed or 0, uniforms=uni)
    else:
        tok, stats = eng.generate_speculative(prompts, new, k, T, seed=useed or 0, uniforms=uni)
    greedy = T <= 0
    exact, ties = compare_tokens(tok, g[f"{name}_tokens"], g[f"{name}_margins"], S, greedy=greedy,
                                 tol=BF16_GREEDY_GAP if greedy else BF16_SAMPLED_MARGIN)
    assert exact + ties == B
    if greedy:
        # greedy forks need a relative top-2 logit gap inside the bf16
        # tolerance: most requests agree with the oracle token for token.
        # Sampled draws over 32000 probabilities sit within the bf16
        # tolerance of a CDF step almost every time, so there the contract
        # is the near-tie rule alone.
        assert exact >= B // 2, (exact, ties)
    if name == "large":
        for e in _ENGINES.values():
            e.close()
        _ENGINES.clear()
