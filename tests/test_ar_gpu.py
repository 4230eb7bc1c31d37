"""Autoregressive decoding on the B200 path (specdec_generate_ar, the
reference's generate_advanced with the KV cache, src/nn/layer.cpp:1239-1380)
against the CPU restatement on identical seeded weights, prompts and
uniforms.  Tokens bit-exact except at logged near-ties
(helpers.compare_tokens): greedy below a 1e-4 relative top-2 logit gap
(2e-2 with bf16 activations), sampled below a 2e-5 distance between the
uniform and a CDF boundary."""
import numpy as np
import pytest

import oracle
import specdec_b200 as sd
from helpers import BF16_GREEDY_GAP, compare_tokens, make_pair
from specdec_b200.synth import ModelShape, make_prompts

pytestmark = pytest.mark.gpu

SHAPES = {
    "tiny8": ModelShape(vocab=8, d_model=8, n_heads=2, d_ff=16, n_layers=2, max_seq_len=96),
    "small": ModelShape(vocab=97, d_model=32, n_heads=4, d_ff=64, n_layers=2, max_seq_len=160),
    "cfg1": ModelShape(vocab=2048, d_model=256, n_heads=4, d_ff=1024, n_layers=4, max_seq_len=200),
}


def _both(pair, B, S, max_new, T, seed=42, top_k=0, top_p=1.0, uniforms=False, prompt_seed=1):
    prompts = make_prompts(B, S, pair.shape.vocab, seed=prompt_seed)
    uni = sd.philox_uniforms(seed, B, max_new, 1) if uniforms else None
    tok_g, st_g = pair.engine.generate_advanced(prompts, max_new, T, top_k, top_p, seed, uniforms=uni)
    tok_o, mg = oracle.oracle_generate_ar(pair.target, prompts, max_new, T, top_k, top_p, seed, uniforms=uni,
                                          act_bf16=pair.act_bf16, kv_mode=pair.kv_mode)
    return prompts, tok_g, st_g, tok_o, mg


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("int8", [False, True])
def test_ar_greedy(gpu_lib, oracle_built, name, int8):
    pair = make_pair(SHAPES[name], 1, seed=5, int8=int8, max_batch=4, max_prompt_len=40)
    prompts, tg, st, to, mg = _both(pair, 3, 17, 40, 0.0)
    exact, ties = compare_tokens(tg, to, mg, 17, greedy=True)
    assert exact + ties == 3 and ties <= 1
    assert (st[:, 0] == 40).all() and (st[:, 1:] == 0).all()


@pytest.mark.parametrize("name", ["small", "cfg1"])
@pytest.mark.parametrize("uniforms", [False, True])
def test_ar_sampled(gpu_lib, oracle_built, name, uniforms):
    pair = make_pair(SHAPES[name], 1, seed=6, int8=True, max_batch=4, max_prompt_len=40)
    prompts, tg, st, to, mg = _both(pair, 4, 21, 48, 1.0, seed=11, uniforms=uniforms)
    exact, ties = compare_tokens(tg, to, mg, 21, greedy=False)
    assert exact + ties == 4 and ties <= 1


def test_ar_top_k_top_p(gpu_lib, oracle_built):
    pair = make_pair(SHAPES["cfg1"], 1, seed=7, max_batch=2, max_prompt_len=40)
    prompts, tg, st, to, mg = _both(pair, 2, 9, 32, 0.9, seed=7, top_k=5, top_p=0.8)
    exact, ties = compare_tokens(tg, to, mg, 9, greedy=False)
    assert exact + ties == 2 and ties <= 1


def test_ar_int8_kv_bf16(gpu_lib, oracle_built):
    pair = make_pair(SHAPES["cfg1"], 1, seed=8, int8=True, act_bf16=True, kv_mode=2, max_batch=2, max_prompt_len=40)
    prompts, tg, st, to, mg = _both(pair, 2, 12, 24, 0.0)
    exact, ties = compare_tokens(tg, to, mg, 12, greedy=True, tol=BF16_GREEDY_GAP)
    assert exact + ties == 2


def test_ar_matches_single_request_reference_stream(gpu_lib, oracle_built):
    # request 0 of a batch with seed s follows generate_advanced(seed = s)
    pair = make_pair(SHAPES["small"], 1, seed=9, max_batch=2, max_prompt_len=40)
    prompts = make_prompts(2, 10, pair.shape.vocab, seed=3)
    tg, _ = pair.engine.generate_advanced(prompts, 20, 0.9, 5, 0.8, 7)
    ref = pair.target.generate_advanced(prompts[0], 20, 0.9, 5, 0.8, 7)
    _, mg = oracle.oracle_generate_ar(pair.target, prompts[:1], 20, 0.9, 5, 0.8, 7)
    compare_tokens(tg[:1], ref[None], mg, 10, greedy=False)


def test_ar_edges(gpu_lib, oracle_built):
    shape = SHAPES["small"]
    pair = make_pair(shape, 1, seed=10, max_batch=2, max_prompt_len=40)
    prompts = make_prompts(2, 6, shape.vocab, seed=4)
    # max_new = 0 returns the prompt; 1 returns the prefill's token
    tg, st = pair.engine.generate_advanced(prompts, 0, 0.0)
    assert np.array_equal(tg, prompts) and (st == 0).all()
    tg, _ = pair.engine.generate_advanced(prompts, 1, 0.0)
    to, _ = oracle.oracle_generate_ar(pair.target, prompts, 1, 0.0)
    assert np.array_equal(tg, to)
    # the cache ends at S + max_new - 1 positions: exactly max_seq_len is fine,
    # one more is the reference's max_seq_len error
    n = shape.max_seq_len - 6 + 1
    tg, _ = pair.engine.generate_advanced(prompts, n, 0.0)
    assert tg.shape == (2, 6 + n)
    with pytest.raises(sd.SpecDecError) as e:
        pair.engine.generate_advanced(prompts, n + 1, 0.0)
    assert e.value.code == 4
    # a uniform table with too few steps
    with pytest.raises(sd.SpecDecError) as e:
        pair.engine.generate_advanced(prompts, 8, 1.0, uniforms=sd.philox_uniforms(1, 2, 4, 1))
    assert e.value.code == 7
    # the engine stays usable after the errors
    tg, _ = pair.engine.generate_advanced(prompts, 5, 0.0)
    to, _ = oracle.oracle_generate_ar(pair.target, prompts, 5, 0.0)
    assert np.array_equal(tg, to)


def test_ar_graph_reuse_and_launch_count(gpu_lib, oracle_built):
    pair = make_pair(SHAPES["cfg1"], 1, seed=11, int8=True, max_batch=4, max_prompt_len=40)
    prompts = make_prompts(4, 16, pair.shape.vocab, seed=5)
    a, _ = pair.engine.generate_advanced(prompts, 30, 0.0)
    b, _ = pair.engine.generate_advanced(prompts, 30, 0.0)  # same graph, replayed
    assert np.array_equal(a, b)
    assert pair.engine.last_launch_count() > 30
