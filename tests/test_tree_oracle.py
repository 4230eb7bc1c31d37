"""Tree speculation in the CPU oracle (no reference counterpart, so parity is
pinned only by these properties): a 1/1/1/1 tree is the k = 4 chain in
greedy mode, any greedy tree reproduces greedy decoding, and the sampled
acceptance rule (top-k children as point-mass proposals, rejected children
zeroed out of p) emits tokens with exactly the target's distribution."""
import numpy as np
import pytest

import oracle
from specdec_b200.synth import ModelShape, draft_params, make_params, make_prompts

SMALL = ModelShape(vocab=97, d_model=32, n_heads=4, d_ff=64, n_layers=2, max_seq_len=160)


def _pair(shape, seed, dl=1):
    P = make_params(shape, seed=seed, bias_std=0.02, ln_jitter=0.05)
    return oracle.Oracle(shape, P), oracle.Oracle(shape.with_layers(dl), draft_params(shape, P, dl))


@pytest.fixture(scope="module")
def small_pair(oracle_built):
    return _pair(SMALL, 31)


def test_tree_chain_equivalence_greedy(small_pair):
    t, d = small_pair
    prompts = make_prompts(3, 12, SMALL.vocab, seed=2)
    tok_c, st_c, _ = oracle.oracle_generate_speculative(t, d, prompts, 30, 4, 0.0, catchup=1)
    tok_t, st_t, _ = oracle.oracle_generate_tree(t, d, prompts, 30, [1, 1, 1, 1], 0.0)
    assert np.array_equal(tok_c, tok_t)
    assert np.array_equal(st_c[:, 0], st_t[:, 0]) and np.array_equal(st_c[:, 2], st_t[:, 2])


def test_tree_greedy_equals_autoregressive(small_pair):
    t, d = small_pair
    prompts = make_prompts(2, 10, SMALL.vocab, seed=3)
    tok_t, st, _ = oracle.oracle_generate_tree(t, d, prompts, 25, [4, 3, 2, 1], 0.0)
    assert st[:, 1].sum() == st[:, 0].sum() * oracle.tree_nodes([4, 3, 2, 1])
    for b in range(2):
        ar = t.generate_advanced(prompts[b], 25, 0.0, 0, 1.0, 1)
        assert np.array_equal(tok_t[b], ar), b


def test_tree_sampled_is_lossless(oracle_built):
    # V = 8: the joint law of the first two generated tokens must be p(t1) p(t2 | t1)
    shape = ModelShape(vocab=8, d_model=8, n_heads=2, d_ff=16, n_layers=2, max_seq_len=64)
    t, d = _pair(shape, 11)
    B, br = 6000, [3, 2]
    prompt = make_prompts(1, 4, 8, seed=5)[0]
    prompts = np.repeat(prompt[None, :], B, axis=0)
    rng = np.random.default_rng(7)
    uni = rng.random((B, 3, oracle.tree_slots(br)), dtype=np.float32)
    tok, _, _ = oracle.oracle_generate_tree(t, d, prompts, 2, br, 1.0, uniforms=uni)
    pairs = tok[:, 4] * 8 + tok[:, 5]
    counts = np.bincount(pairs, minlength=64).astype(np.float64)
    p1 = oracle.oracle_get_probs(t.forward(prompt)[-1], 1.0)
    expect = np.zeros(64)
    for a in range(8):
        p2 = oracle.oracle_get_probs(t.forward(np.append(prompt, a))[-1], 1.0)
        expect[a * 8:(a + 1) * 8] = p1[a] * p2
    expect *= B
    keep = expect > 5
    chi2 = float(((counts[keep] - expect[keep]) ** 2 / expect[keep]).sum())
    dof = int(keep.sum()) - 1
    # 99.9 % quantile of chi-square with dof degrees of freedom (Wilson-Hilferty)
    z = 3.09
    crit = dof * (1 - 2 / (9 * dof) + z * np.sqrt(2 / (9 * dof))) ** 3
    assert chi2 < crit, (chi2, crit, dof)
