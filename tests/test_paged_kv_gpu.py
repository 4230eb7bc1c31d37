"""The paged KV cache against the CPU oracle.

The reference's KVCache (include/nn/layer.hpp:212-230) holds one contiguous
tensor per layer and grows it by copying (src/nn/layer.cpp:667-809); here
each model's cache is a pool of 128-position pages and every request has a
page table.  A call takes the pages its requests can reach (prompt + new
tokens + one verify block, and up to new positions more: under the reference
catch-up the draft is fed one extra position per rejected round, so its cache
runs ahead of the target's): request b's i-th page is the pool's (i*B + b)-th,
so a request's pages are never adjacent once B > 1, and every multi-request
test of the suite runs on scattered pages.  These cases add pools sized to
the call (not to max_seq_len), caches that cross several pages, the three
cache types and both attention families, and the pool-exhausted error."""
import numpy as np
import pytest

import oracle
import specdec_b200 as sd
from helpers import BF16_GREEDY_GAP, compare_tokens, make_pair
from specdec_b200.synth import ModelShape, make_prompts

pytestmark = pytest.mark.gpu

PAGE = 128
D64 = ModelShape(vocab=2048, d_model=256, n_heads=4, d_ff=1024, n_layers=2, max_seq_len=1024)
D128 = ModelShape(vocab=2048, d_model=512, n_heads=4, d_ff=1024, n_layers=2, max_seq_len=1024)


def pages_for(B, S, new, k):
    # prompt + new tokens + a verify block, and the draft cache's drift under
    # the reference catch-up (one position per rejected round, at most new)
    return B * -(-(S + 2 * new + k + 1) // PAGE)


# (shape, int8 weights, bf16 activations, kv mode): fp32 cache with the
# CUDA-core attention, bf16 cache with the tensor-core prefill attention
# (head_dim 64) or the decode kernel (head_dim 128), int8 cache with its
# per-row scale planes
CASES = [
    ("d64", False, False, 0),
    ("d64", True, True, 1),
    ("d128", True, True, 1),
    ("d64", True, False, 2),
]


@pytest.mark.parametrize("shape,int8,bf16,kv", CASES)
@pytest.mark.parametrize("greedy", [True, False])
def test_call_sized_pool_matches_oracle(gpu_lib, oracle_built, shape, int8, bf16, kv, greedy):
    """A pool of exactly the pages the call needs (not max_batch x
    max_seq_len): prompts of 300 positions cross into a third page and the
    generation into a fourth; tokens match the oracle and the default pool."""
    m = D64 if shape == "d64" else D128
    B, S, new, k = 3, 300, 60, 4
    need = pages_for(B, S, new, k)
    assert need < B * -(-m.max_seq_len // PAGE)
    small = make_pair(m, 1, seed=51, int8=int8, act_bf16=bf16, kv_mode=kv, max_batch=B, max_prompt_len=S,
                      kv_pages=need)
    full = make_pair(m, 1, seed=51, int8=int8, act_bf16=bf16, kv_mode=kv, max_batch=B, max_prompt_len=S)
    prompts = make_prompts(B, S, m.vocab, seed=6)
    T = 0.0 if greedy else 1.0
    uni = None if greedy else sd.philox_uniforms(91, B, new + 2, 2 * k + 1)
    ts, ss = small.engine.generate_speculative(prompts, new, k, T, seed=91, uniforms=uni)
    tf, sf = full.engine.generate_speculative(prompts, new, k, T, seed=91, uniforms=uni)
    assert np.array_equal(ts, tf) and np.array_equal(ss, sf)
    to, _, mg = oracle.oracle_generate_speculative(small.target, small.draft, prompts, new, k, T, seed=91,
                                                   uniforms=uni, act_bf16=bf16, kv_mode=kv,
                                                   cache_cap=m.max_seq_len)
    tol = (BF16_GREEDY_GAP if bf16 else None) if greedy else 2e-3
    compare_tokens(ts, to, mg, S, greedy=greedy, tol=tol)
    small.engine.close()
    full.engine.close()


def test_session_on_call_sized_pool(gpu_lib, oracle_built):
    """The round-level session keeps its pages across steps."""
    B, S, new, k = 2, 250, 40, 4
    pair = make_pair(D64, 1, seed=52, int8=True, max_batch=B, max_prompt_len=S, kv_pages=pages_for(B, S, new, k))
    prompts = make_prompts(B, S, D64.vocab, seed=7)
    want, _ = pair.engine.generate_speculative(prompts, new, k, 0.0)
    pair.engine.prefill(prompts, new, k, 0.0)
    for _ in range(new):
        pair.engine.step(1)
    got, _ = pair.engine.session_tokens()
    assert np.array_equal(got, want)
    pair.engine.close()


def test_draft_drift_within_pages(gpu_lib, oracle_built):
    """A long generation with a draft that is rarely accepted: under the
    reference catch-up the draft cache drifts ahead of the target's by one
    position per rejected round (here well past one page), and the call's
    pages still cover it; tokens match the default pool and the oracle."""
    B, S, new, k = 2, 100, 200, 4
    small = make_pair(D64, 1, seed=53, int8=True, max_batch=B, max_prompt_len=S, kv_pages=pages_for(B, S, new, k))
    full = make_pair(D64, 1, seed=53, int8=True, max_batch=B, max_prompt_len=S)
    prompts = make_prompts(B, S, D64.vocab, seed=12)
    ts, ss = small.engine.generate_speculative(prompts, new, k, 0.0)
    tf, sf = full.engine.generate_speculative(prompts, new, k, 0.0)
    assert np.array_equal(ts, tf) and np.array_equal(ss, sf)
    to, _, mg = oracle.oracle_generate_speculative(small.target, small.draft, prompts, new, k, 0.0,
                                                   cache_cap=D64.max_seq_len)
    compare_tokens(ts, to, mg, S, greedy=True)
    small.engine.close()
    full.engine.close()


def test_pool_exhausted(gpu_lib):
    """More pages than the pool holds: SPECDEC_ERR_OOM before any launch;
    a call that fits still runs afterwards."""
    from specdec_b200.synth import make_params

    eng = sd.Engine(D64, draft_layers=1, max_batch=4, max_prompt_len=256, kv_pages=6)
    eng.load_params(sd.TARGET, make_params(D64, seed=3))
    prompts = make_prompts(4, 200, D64.vocab, seed=8)  # 4 requests x 2 pages > 6
    with pytest.raises(sd.SpecDecError) as e:
        eng.generate_speculative(prompts, 20, 4, 0.0)
    assert e.value.code == 3 and "page pool" in str(e.value)
    with pytest.raises(sd.SpecDecError) as e:
        eng.prefill(prompts, 20, 4, 0.0)
    assert e.value.code == 3
    toks, _ = eng.generate_speculative(prompts[:3], 20, 4, 0.0)  # 3 x 2 pages fit
    assert toks.shape == (3, 220)
    eng.close()
