"""Tensor-core decode / verify attention for head_dim 128 (csrc/attn_dec.cu)
against the CPU oracle and against the CUDA-core attention kernel.

The kernel serves groups of at most 16 query rows over a bf16 cache with
head_dim 128 (the large configuration's 32 heads x 128): draft steps, the
(k+1)-row verify block and short forwards.  Its splits (several CTAs over one
request's cache, merged by the last one to finish) engage when few
(request, head) items would leave SMs idle, so the long-context cases here
run with split merges, and the batched ones without.

Tolerances as the parity contract states them for bf16 activations: logits
within 2e-2 relative; tokens bit-exact except at near-ties of the oracle's
decision margins (helpers.compare_tokens)."""
import os

import numpy as np
import pytest

import oracle
import specdec_b200 as sd
from helpers import BF16_GREEDY_GAP, compare_tokens, make_pair
from specdec_b200.synth import ModelShape, make_prompts

pytestmark = pytest.mark.gpu

BF16_REL = 2e-2
# The two attention kernels differ only in summation order and the bf16
# rounding of probabilities before P.V
KERNEL_REL = 1e-2

D128 = ModelShape(vocab=2048, d_model=512, n_heads=4, d_ff=1024, n_layers=2, max_seq_len=2048)


def rel_err(a, b):
    return float(np.max(np.abs(a - b)) / max(1e-30, float(np.max(np.abs(b)))))


def _pair(env_dec: str, **kw):
    old = os.environ.get("SPECDEC_ATTN_DEC")
    os.environ["SPECDEC_ATTN_DEC"] = env_dec
    try:
        return make_pair(D128, 1, seed=21, int8=True, act_bf16=True, kv_mode=1, **kw)
    finally:
        if old is None:
            del os.environ["SPECDEC_ATTN_DEC"]
        else:
            os.environ["SPECDEC_ATTN_DEC"] = old


@pytest.mark.parametrize("S", [1, 5, 16])
def test_forward_logits_d128(gpu_lib, oracle_built, S):
    """One group of S <= 16 rows: the decode kernel (one (group, head) per
    head: split over the cache), vs the oracle and the CUDA-core kernel."""
    on = _pair("1", max_prompt_len=64, max_batch=2)
    off = _pair("0", max_prompt_len=64, max_batch=2)
    toks = make_prompts(1, S, D128.vocab, seed=40 + S)[0]
    for role, om in ((sd.TARGET, on.target), (sd.DRAFT, on.draft)):
        g = on.engine.forward_logits(role, toks)
        c = off.engine.forward_logits(role, toks)
        o = om.forward(toks, act_bf16=True, kv_mode=1)
        assert rel_err(g, o) < BF16_REL, (S, role, rel_err(g, o))
        assert rel_err(g, c) < KERNEL_REL, (S, role, rel_err(g, c))
    on.engine.close()
    off.engine.close()


@pytest.mark.parametrize("greedy", [True, False])
def test_spec_long_context_d128(gpu_lib, oracle_built, greedy):
    """Speculative decoding after a 1200-token prompt: every draft step and
    verify block runs the decode kernel with split merges (2 requests x 4
    heads = 8 items, ten 128-position tiles each)."""
    B, S, new, k = 2, 1200, 24, 4
    pair = _pair("1", max_prompt_len=S, max_batch=B)
    prompts = make_prompts(B, S, D128.vocab, seed=3)
    T = 0.0 if greedy else 1.0
    uni = None if greedy else sd.philox_uniforms(77, B, new + 2, 2 * k + 1)
    tok_g, _ = pair.engine.generate_speculative(prompts, new, k, T, seed=77, uniforms=uni)
    tok_o, _, mg = oracle.oracle_generate_speculative(pair.target, pair.draft, prompts, new, k, T, seed=77,
                                                      uniforms=uni, act_bf16=True, kv_mode=1,
                                                      cache_cap=D128.max_seq_len)
    compare_tokens(tok_g, tok_o, mg, S, greedy=greedy, tol=BF16_GREEDY_GAP if greedy else 2e-3)
    pair.engine.close()


def test_spec_batched_d128_kernels_agree(gpu_lib, oracle_built):
    """16 requests x 4 heads: enough (request, head) items that the decode
    kernel does not split; the same generation with the CUDA-core kernel
    gives the same greedy tokens except at near-ties."""
    B, S, new, k = 16, 96, 16, 4
    on = _pair("1", max_prompt_len=S, max_batch=B)
    off = _pair("0", max_prompt_len=S, max_batch=B)
    prompts = make_prompts(B, S, D128.vocab, seed=5)
    tg, _ = on.engine.generate_speculative(prompts, new, k, 0.0)
    tc, _ = off.engine.generate_speculative(prompts, new, k, 0.0)
    to, _, mg = oracle.oracle_generate_speculative(on.target, on.draft, prompts, new, k, 0.0, act_bf16=True,
                                                   kv_mode=1, cache_cap=D128.max_seq_len)
    compare_tokens(tg, to, mg, S, greedy=True, tol=BF16_GREEDY_GAP)
    compare_tokens(tc, to, mg, S, greedy=True, tol=BF16_GREEDY_GAP)
    on.engine.close()
    off.engine.close()


@pytest.mark.parametrize("S", [16, 40, 96, 160, 256])
def test_gemm_w8_forward(gpu_lib, oracle_built, S):
    """The int8-code tensor-core GEMM (csrc/gemm_w8.cu: features on the MMA's
    M side, rows on N; opt-in with SPECDEC_GEMM_W8=1) at row counts from a
    draft step to its 256-row limit, against the oracle and against the
    bf16-image GEMM / GEMV path."""
    old = os.environ.get("SPECDEC_GEMM_W8")
    try:
        os.environ["SPECDEC_GEMM_W8"] = "0"
        off = make_pair(D128, 1, seed=22, int8=True, act_bf16=True, kv_mode=1, max_prompt_len=256, max_batch=2)
        os.environ["SPECDEC_GEMM_W8"] = "1"
        on = make_pair(D128, 1, seed=22, int8=True, act_bf16=True, kv_mode=1, max_prompt_len=256, max_batch=2)
    finally:
        if old is None:
            del os.environ["SPECDEC_GEMM_W8"]
        else:
            os.environ["SPECDEC_GEMM_W8"] = old
    toks = make_prompts(1, S, D128.vocab, seed=60 + S)[0]
    for role, om in ((sd.TARGET, on.target), (sd.DRAFT, on.draft)):
        g = on.engine.forward_logits(role, toks)
        c = off.engine.forward_logits(role, toks)
        o = om.forward(toks, act_bf16=True, kv_mode=1)
        assert rel_err(g, o) < BF16_REL, (S, role, rel_err(g, o))
        assert rel_err(g, c) < KERNEL_REL, (S, role, rel_err(g, c))
    on.engine.close()
    off.engine.close()
