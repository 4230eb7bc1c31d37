"""The round-level session (specdec_prefill / specdec_step /
specdec_session_tokens): generate_speculative split at its round loop
(src/nn/layer.cpp:1514-1656) gives the same tokens as the whole generation
and as the oracle, whether the rounds run one per call or several, and
whether the host uniforms come with the prefill or with each step."""
import numpy as np
import pytest

import oracle
import specdec_b200 as sd
from helpers import compare_tokens, make_pair, run_both
from specdec_b200.synth import ModelShape, make_prompts

pytestmark = pytest.mark.gpu

CFG1 = ModelShape(vocab=2048, d_model=256, n_heads=4, d_ff=1024, n_layers=4, max_seq_len=200)


def _run_session(eng, prompts, new, k, T, seed, uni, rounds_per_call, per_step_uniforms=False):
    B = prompts.shape[0]
    if per_step_uniforms:
        # the prefill only brings round 0 (the first token); each step brings its own rounds
        eng.prefill(prompts, new, k, T, seed=seed, uniforms=np.ascontiguousarray(uni[:, :1]))
    else:
        eng.prefill(prompts, new, k, T, seed=seed, uniforms=uni)
    emitted = [[] for _ in range(B)]
    r = 1
    for _ in range(new + 2):
        u = np.ascontiguousarray(uni[:, r:r + rounds_per_call]) if per_step_uniforms else None
        if u is not None and u.shape[1] < rounds_per_call:
            break
        toks, cnt = eng.step(rounds_per_call, uniforms=u)
        r += rounds_per_call
        for b in range(B):
            assert 0 <= cnt[b] <= rounds_per_call * (k + 1)
            emitted[b].extend(toks[b, :cnt[b]].tolist())
        if all(len(e) >= new - 1 for e in emitted):
            break
    full, stats = eng.session_tokens()
    return full, stats, emitted


@pytest.mark.parametrize("rounds_per_call", [1, 3])
@pytest.mark.parametrize("per_step_uniforms", [False, True])
def test_session_equals_generate(gpu_lib, oracle_built, rounds_per_call, per_step_uniforms):
    pair = make_pair(CFG1, 1, seed=31, int8=True, max_batch=3, max_prompt_len=24)
    B, S, new, k = 3, 20, 30, 4
    prompts = make_prompts(B, S, CFG1.vocab, seed=8)
    uni = sd.philox_uniforms(5, B, new + 2, 2 * k + 1)
    want, wstats = pair.engine.generate_speculative(prompts, new, k, 1.0, seed=5, uniforms=uni)
    full, stats, emitted = _run_session(pair.engine, prompts, new, k, 1.0, 5, uni, rounds_per_call,
                                        per_step_uniforms)
    assert np.array_equal(full, want)
    assert np.array_equal(stats, wstats)
    for b in range(B):
        # the first new token comes from the prefill, the rest from the steps
        assert emitted[b] == want[b, S + 1:].tolist()
    pair.engine.close()


def test_session_greedy_matches_oracle(gpu_lib, oracle_built):
    pair = make_pair(CFG1, 1, seed=32, max_batch=2, max_prompt_len=24)
    B, S, new, k = 2, 16, 25, 4
    prompts = make_prompts(B, S, CFG1.vocab, seed=9)
    pair.engine.prefill(prompts, new, k, 0.0)
    for _ in range(new):
        pair.engine.step(1)
    full, _ = pair.engine.session_tokens()
    ref, _, mg = oracle.oracle_generate_speculative(pair.target, pair.draft, prompts, new, k, 0.0,
                                                    cache_cap=CFG1.max_seq_len)
    compare_tokens(full, ref, mg, S, greedy=True)
    pair.engine.close()


def test_session_call_order(gpu_lib):
    from specdec_b200.synth import make_params

    eng = sd.Engine(CFG1, draft_layers=1, max_batch=2, max_prompt_len=16)
    eng.load_params(sd.TARGET, make_params(CFG1, seed=1))
    eng._session = (2, 8, 4, 10)
    with pytest.raises(sd.SpecDecError) as e:
        eng.step(1)
    assert e.value.code == 6  # no open session
    prompts = make_prompts(2, 8, CFG1.vocab, seed=1)
    eng.prefill(prompts, 10, 4, 0.0)
    with pytest.raises(sd.SpecDecError) as e:
        eng.step(0)
    assert e.value.code == 1
    eng.step(2)
    # a whole generation closes the session
    eng.generate_speculative(prompts, 4, 4, 0.0)
    with pytest.raises(sd.SpecDecError) as e:
        eng.step(1)
    assert e.value.code == 6
    eng.close()


@pytest.mark.parametrize("int8,bf16", [(False, False), (True, False), (True, True)])
def test_load_params_device_equals_host(gpu_lib, int8, bf16):
    """specdec_load_params_device (scales, codes and transpose on the GPU)
    gives the same device parameters as the host loader: identical logits."""
    import torch

    from specdec_b200.synth import make_params

    shape = ModelShape(vocab=384, d_model=128, n_heads=2, d_ff=352, n_layers=2, max_seq_len=64)
    P = make_params(shape, seed=41, bias_std=0.02, ln_jitter=0.05)
    kw = dict(weight_dtype=sd.INT8 if int8 else sd.F32, act_dtype=sd.BF16 if bf16 else sd.F32,
              kv_dtype=sd.BF16 if bf16 else sd.F32, max_batch=2, max_prompt_len=64)
    host = sd.Engine(shape, draft_layers=1, **kw)
    host.load_params(sd.TARGET, P)
    dev = sd.Engine(shape, draft_layers=1, **kw)
    dev.load_params_device(sd.TARGET, [torch.from_numpy(np.ascontiguousarray(p, np.float32)).cuda() for p in P])
    toks = make_prompts(1, 40, shape.vocab, seed=2)[0]
    for role in (sd.TARGET, sd.DRAFT):
        assert np.array_equal(host.forward_logits(role, toks), dev.forward_logits(role, toks))
    host.close()
    dev.close()
