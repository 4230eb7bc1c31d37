"""The reference-side binding, compiled and run: the reference library built
from its own sources with the dispatch a maintainer would add
(oracle/binding/cuda_spec_backend.*, inserted into src/nn/layer.cpp by
oracle/bind_reference.py; oracle/_ref/libnnref_cuda.so), linked to
libspecdec_b200.so.  A TransformerDecoder constructed on a CudaSpecBackend
answers the UNCHANGED generate_speculative and generate_advanced
(include/nn/layer.hpp:312-323) from the device, and the tokens equal those of
the stock reference library (oracle/_ref/libnnref.so) on the same weights:
greedy exactly, quantized_cache = true through the int8 cache, sampled
(the reference's std::mt19937(seed) stream) up to the near-ties of the
oracle's decision margins."""
import numpy as np
import pytest

import oracle
from helpers import GREEDY_REL_GAP, SAMPLED_MARGIN, compare_tokens
from specdec_b200.synth import ModelShape, draft_params, make_params, make_prompts

pytestmark = pytest.mark.gpu

SHAPE = ModelShape(vocab=512, d_model=128, n_heads=4, d_ff=256, n_layers=3, max_seq_len=128)


@pytest.fixture(scope="module")
def models(gpu_lib, oracle_built):
    assert oracle.bound_reference_available(), "oracle/_ref/libnnref_cuda.so is missing (make -C oracle bind)"
    P = make_params(SHAPE, seed=71, bias_std=0.02, ln_jitter=0.05)
    DP = draft_params(SHAPE, P, 1)
    stock = (oracle.Reference(SHAPE, P, requires_grad=False),
             oracle.Reference(SHAPE.with_layers(1), DP, requires_grad=False))
    be = oracle.CudaSpecBackendRef(SHAPE, SHAPE.with_layers(1))
    bound = (oracle.Reference(SHAPE, P, requires_grad=False, backend=be),
             oracle.Reference(SHAPE.with_layers(1), DP, requires_grad=False, backend=be))
    restated = (oracle.Oracle(SHAPE, P), oracle.Oracle(SHAPE.with_layers(1), DP))
    yield stock, bound, restated, be
    del bound
    be.close()


@pytest.mark.parametrize("quantized_cache", [False, True])
def test_generate_speculative_greedy(models, quantized_cache):
    stock, bound, _, be = models
    for i in range(3):
        prompt = make_prompts(1, 12 + 5 * i, SHAPE.vocab, seed=80 + i)[0]
        want = stock[0].generate_speculative(stock[1], prompt, 40, 4, 0.0, quantized_cache=quantized_cache)
        got = bound[0].generate_speculative(bound[1], prompt, 40, 4, 0.0, quantized_cache=quantized_cache)
        assert be.launches() != 0  # the call ran on the device
        # a token may differ only where the restatement's own decision
        # margin (relative top-2 logit gap) is a near-tie; with the int8 cache
        # the tolerance is that of its per-(position, head) rounding
        _, _, mg = oracle.oracle_generate_speculative(models[2][0], models[2][1], prompt[None], 40, 4, 0.0,
                                                      kv_mode=2 if quantized_cache else 0,
                                                      cache_cap=SHAPE.max_seq_len)
        compare_tokens(np.array(got)[None], np.array(want)[None], mg, prompt.size, greedy=True,
                       tol=1e-2 if quantized_cache else GREEDY_REL_GAP)


def test_generate_speculative_sampled(models):
    stock, bound, restated, be = models
    for i in range(3):
        prompt = make_prompts(1, 16, SHAPE.vocab, seed=90 + i)[0]
        want = stock[0].generate_speculative(stock[1], prompt, 32, 4, 1.0, 0, 1.0, 1000 + i)
        got = bound[0].generate_speculative(bound[1], prompt, 32, 4, 1.0, 0, 1.0, 1000 + i)
        _, _, mg = oracle.oracle_generate_speculative(restated[0], restated[1], prompt[None], 32, 4, 1.0,
                                                      seed=1000 + i, cache_cap=SHAPE.max_seq_len)
        compare_tokens(np.array(got)[None], np.array(want)[None], mg, prompt.size, greedy=False, tol=SAMPLED_MARGIN)


def test_generate_advanced(models):
    stock, bound, _, be = models
    for T, seed in ((0.0, 1), (1.0, 7)):
        prompt = make_prompts(1, 10, SHAPE.vocab, seed=95)[0]
        want = stock[0].generate_advanced(prompt, 30, T, 0, 1.0, seed)
        got = bound[0].generate_advanced(prompt, 30, T, 0, 1.0, seed)
        assert be.launches() != 0
        _, mg = oracle.oracle_generate_ar(models[2][0], prompt[None], 30, T, seed=seed)
        compare_tokens(np.array(got)[None], np.array(want)[None], mg, prompt.size, greedy=T <= 0)
    # use_kv_cache = false stays on the host path of the same library
    prompt = make_prompts(1, 10, SHAPE.vocab, seed=96)[0]
    assert list(bound[0].generate_advanced(prompt, 8, 0.0, use_kv_cache=False)) == \
        list(stock[0].generate_advanced(prompt, 8, 0.0, use_kv_cache=False))
