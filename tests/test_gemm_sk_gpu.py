"""The persistent stream-K GEMM (csrc/gemm_sk.cu) against the oracle and
against the cluster split-K GEMM.

The engine sends row batches of at most 256 rows over layers of at least
SPECDEC_SK_MIN_TILES 256-column tiles to it (80 by default: the large
config's gate/up and lm_head).  With the threshold at 1 every GEMM
launch of this small model takes it, so each tile is shared by several CTAs
(8-16 k-blocks per tile, one or two per CTA) and every output goes through the
fix-up of partial tiles; 129-256 rows use both 128-row accumulators.

Tolerances as for every bf16 path: logits within 2e-2 of the oracle, 1e-2
between the two GEMMs (only the fp32 summation order differs); greedy tokens
bit-exact except at near-ties."""
import os

import numpy as np
import pytest

import oracle
import specdec_b200 as sd
from helpers import BF16_GREEDY_GAP, compare_tokens, make_pair
from specdec_b200.synth import ModelShape, make_prompts

pytestmark = pytest.mark.gpu

BF16_REL = 2e-2
KERNEL_REL = 1e-2
SHAPE = ModelShape(vocab=2048, d_model=512, n_heads=4, d_ff=1024, n_layers=2, max_seq_len=512)


def rel_err(a, b):
    return float(np.max(np.abs(a - b)) / max(1e-30, float(np.max(np.abs(b)))))


def _pair(sk: bool, **kw):
    saved = {k: os.environ.get(k) for k in ("SPECDEC_GEMM_SK", "SPECDEC_SK_MIN_TILES")}
    os.environ["SPECDEC_GEMM_SK"] = "1" if sk else "0"
    os.environ["SPECDEC_SK_MIN_TILES"] = "1"
    try:
        return make_pair(SHAPE, 1, seed=23, int8=True, act_bf16=True, kv_mode=1, **kw)
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


@pytest.mark.parametrize("S", [64, 100, 128, 129, 200, 256])
def test_gemm_sk_forward(gpu_lib, oracle_built, S):
    on = _pair(True, max_prompt_len=256, max_batch=2)
    off = _pair(False, max_prompt_len=256, max_batch=2)
    toks = make_prompts(1, S, SHAPE.vocab, seed=70 + S)[0]
    for role, om in ((sd.TARGET, on.target), (sd.DRAFT, on.draft)):
        g = on.engine.forward_logits(role, toks)
        c = off.engine.forward_logits(role, toks)
        o = om.forward(toks, act_bf16=True, kv_mode=1)
        assert rel_err(g, o) < BF16_REL, (S, role, rel_err(g, o))
        assert rel_err(g, c) < KERNEL_REL, (S, role, rel_err(g, c))
        # the fix-up adds the pieces in a fixed order: the same bits every run
        assert np.array_equal(g, on.engine.forward_logits(role, toks))
    on.engine.close()
    off.engine.close()


@pytest.mark.parametrize("B", [16, 40])
def test_gemm_sk_generation(gpu_lib, oracle_built, B):
    """Speculative decoding with every verify block (B x 5 rows: 80 or 200)
    on the stream-K GEMM: greedy tokens match the oracle, and a second run
    gives the same tokens."""
    S, new, k = 48, 24, 4
    pair = _pair(True, max_prompt_len=S, max_batch=B)
    prompts = make_prompts(B, S, SHAPE.vocab, seed=11)
    t1, _ = pair.engine.generate_speculative(prompts, new, k, 0.0)
    t2, _ = pair.engine.generate_speculative(prompts, new, k, 0.0)
    assert np.array_equal(t1, t2)
    to, _, mg = oracle.oracle_generate_speculative(pair.target, pair.draft, prompts, new, k, 0.0, act_bf16=True,
                                                   kv_mode=1, cache_cap=SHAPE.max_seq_len)
    compare_tokens(t1, to, mg, S, greedy=True, tol=BF16_GREEDY_GAP)
    pair.engine.close()
