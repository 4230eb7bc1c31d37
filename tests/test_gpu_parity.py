"""Parity of the B200 path (through the C ABI) against the CPU restatement
oracle on identical seeded weights, prompts and uniforms.

Tolerances (the ones the parity contract states): logits within 1e-3
relative in fp32 and 2e-2 relative with bf16 activations; tokens bit-exact
except at logged near-ties (helpers.compare_tokens)."""
import numpy as np
import pytest

import oracle
import specdec_b200 as sd
from helpers import BF16_GREEDY_GAP, compare_tokens, make_pair, run_both
from specdec_b200.synth import ARCH_CFG, ModelShape, make_prompts

pytestmark = pytest.mark.gpu

FP32_REL = 1e-3
BF16_REL = 2e-2

SHAPES = {
    "tiny8": (ModelShape(vocab=8, d_model=8, n_heads=2, d_ff=16, n_layers=2, max_seq_len=96), 1),
    "small": (ModelShape(vocab=97, d_model=32, n_heads=4, d_ff=64, n_layers=2, max_seq_len=160), 1),
    "cfg1": (ModelShape(vocab=2048, d_model=256, n_heads=4, d_ff=1024, n_layers=4, max_seq_len=200), 1),
}


def rel_err(a, b):
    return float(np.max(np.abs(a - b)) / max(1e-30, float(np.max(np.abs(b)))))


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("int8", [False, True])
def test_forward_logits(gpu_lib, oracle_built, name, int8):
    shape, dl = SHAPES[name]
    pair = make_pair(shape, dl, seed=3, int8=int8, max_prompt_len=40)
    toks = make_prompts(1, 33, shape.vocab, seed=9)[0]
    for role, om in ((sd.TARGET, pair.target), (sd.DRAFT, pair.draft)):
        g = pair.engine.forward_logits(role, toks)
        o = om.forward(toks)
        assert rel_err(g, o) < FP32_REL, (name, role, rel_err(g, o))


def test_forward_logits_bf16(gpu_lib, oracle_built):
    shape, dl = SHAPES["cfg1"]
    pair = make_pair(shape, dl, seed=4, int8=True, act_bf16=True, kv_mode=1, max_prompt_len=40)
    toks = make_prompts(1, 24, shape.vocab, seed=10)[0]
    g = pair.engine.forward_logits(sd.TARGET, toks)
    o = pair.target.forward(toks, act_bf16=True, kv_mode=1)
    assert rel_err(g, o) < BF16_REL


@pytest.mark.parametrize("name", ["tiny8", "small", "cfg1"])
@pytest.mark.parametrize("int8", [False, True])
def test_forward_logits_short(gpu_lib, oracle_built, name, int8):
    # short inputs, down to a single token
    shape, dl = SHAPES[name]
    pair = make_pair(shape, dl, seed=12, int8=int8, max_prompt_len=40)
    for S in (1, 5, 16):
        toks = make_prompts(1, S, shape.vocab, seed=20 + S)[0]
        for role, om in ((sd.TARGET, pair.target), (sd.DRAFT, pair.draft)):
            g = pair.engine.forward_logits(role, toks)
            o = om.forward(toks)
            assert rel_err(g, o) < FP32_REL, (name, S, role, rel_err(g, o))


def test_forward_logits_cfg_arch(gpu_lib, oracle_built):
    shape = ModelShape(vocab=300, d_model=64, n_heads=4, d_ff=128, n_layers=3, max_seq_len=64, arch=ARCH_CFG)
    pair = make_pair(shape, 1, seed=5, max_prompt_len=40)
    toks = make_prompts(1, 20, shape.vocab, seed=11)[0]
    for role, om in ((sd.TARGET, pair.target), (sd.DRAFT, pair.draft)):
        assert rel_err(pair.engine.forward_logits(role, toks), om.forward(toks)) < FP32_REL


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("B", [1, 3])
def test_greedy_spec(gpu_lib, oracle_built, name, B):
    shape, dl = SHAPES[name]
    pair = make_pair(shape, dl, seed=6, max_batch=4, max_prompt_len=40)
    _, tg, sg, to, so, mg = run_both(pair, B, 12, 40, 4, 0.0)
    exact, ties = compare_tokens(tg, to, mg, 12, greedy=True)
    assert exact + ties == B and ties <= max(1, B // 3)
    if ties == 0:
        assert np.array_equal(sg, so)


@pytest.mark.parametrize("name", ["tiny8", "small", "cfg1"])
@pytest.mark.parametrize("T", [1.0, 0.7])
def test_sampled_mt19937(gpu_lib, oracle_built, name, T):
    shape, dl = SHAPES[name]
    pair = make_pair(shape, dl, seed=7, max_batch=4, max_prompt_len=40)
    _, tg, sg, to, so, mg = run_both(pair, 3, 10, 48, 3, T, seed=123)
    exact, ties = compare_tokens(tg, to, mg, 10, greedy=False)
    assert exact + ties == 3 and ties <= 1


def test_sampled_mt19937_long(gpu_lib, oracle_built):
    # enough draws that every request's MT19937 state is regenerated several
    # times, including draws that end exactly on the state's last word
    shape, dl = SHAPES["small"]
    pair = make_pair(shape, dl, seed=13, max_batch=4, max_prompt_len=40)
    _, tg, sg, to, so, mg = run_both(pair, 3, 8, 140, 3, 1.0, seed=77)
    exact, ties = compare_tokens(tg, to, mg, 8, greedy=False)
    assert exact + ties == 3 and ties <= 1


@pytest.mark.parametrize("int8", [False, True])
def test_sampled_host_uniforms(gpu_lib, oracle_built, int8):
    shape, dl = SHAPES["cfg1"]
    pair = make_pair(shape, dl, seed=8, int8=int8, max_batch=4, max_prompt_len=40)
    _, tg, sg, to, so, mg = run_both(pair, 4, 16, 48, 4, 1.0, seed=2024, use_uniforms=True)
    exact, ties = compare_tokens(tg, to, mg, 16, greedy=False)
    assert exact + ties == 4 and ties <= 1


@pytest.mark.parametrize("T", [0.0, 1.0])
def test_catchup_correct(gpu_lib, oracle_built, T):
    shape, dl = SHAPES["small"]
    pair = make_pair(shape, dl, seed=9, max_batch=4, max_prompt_len=40)
    _, tg, sg, to, so, mg = run_both(pair, 2, 8, 40, 3, T, seed=5, use_uniforms=T > 0, catchup=1)
    exact, ties = compare_tokens(tg, to, mg, 8, greedy=T <= 0)
    assert exact + ties == 2


# get_probs top-k / top-p filtering (src/nn/layer.cpp:1451-1471) on the device
# sampler: both uniform sources, filters alone and combined.
@pytest.mark.parametrize("name", ["small", "cfg1"])
@pytest.mark.parametrize("top_k,top_p", [(5, 1.0), (0, 0.8), (40, 0.9), (3, 0.5)])
@pytest.mark.parametrize("use_uniforms", [False, True])
def test_sampled_topk_topp(gpu_lib, oracle_built, name, top_k, top_p, use_uniforms):
    shape, dl = SHAPES[name]
    pair = make_pair(shape, dl, seed=12, max_batch=4, max_prompt_len=40)
    _, tg, sg, to, so, mg = run_both(pair, 3, 10, 40, 3, 0.9, seed=77, use_uniforms=use_uniforms,
                                     top_k=top_k, top_p=top_p)
    exact, ties = compare_tokens(tg, to, mg, 10, greedy=False)
    assert exact + ties == 3 and ties <= 1


# Head dims whose cache rows take the other TMA swizzle spans: D=16 (int8 rows
# of 16 bytes: no swizzle; fp32 64 bytes: 64B), D=32 (int8 32 bytes: 32B;
# bf16 64 bytes: 64B; fp32 128 bytes: 128B).
SWZ_SHAPES = {
    "d16": (ModelShape(vocab=300, d_model=64, n_heads=4, d_ff=128, n_layers=2, max_seq_len=96), 1),
    "d32": (ModelShape(vocab=300, d_model=128, n_heads=4, d_ff=256, n_layers=2, max_seq_len=96), 1),
}
SHAPES_KV = {**SWZ_SHAPES, "cfg1": SHAPES["cfg1"]}


@pytest.mark.parametrize("name", list(SWZ_SHAPES))
@pytest.mark.parametrize("kv_mode", [0, 1])
def test_forward_logits_swizzle_spans(gpu_lib, oracle_built, name, kv_mode):
    shape, dl = SWZ_SHAPES[name]
    pair = make_pair(shape, dl, seed=16, kv_mode=kv_mode, max_prompt_len=64)
    toks = make_prompts(1, 57, shape.vocab, seed=17)[0]
    g = pair.engine.forward_logits(sd.TARGET, toks)
    o = pair.target.forward(toks, kv_mode=kv_mode)
    assert rel_err(g, o) < (FP32_REL if kv_mode == 0 else BF16_REL)


# int8 KV cache (quantize_kv, src/nn/layer.cpp:635-665): per (position, kv
# head) absmax scales, dequantised inside attention.  Rows must be at least
# 16 bytes (head_dim >= 16).
@pytest.mark.parametrize("name", list(SHAPES_KV))
def test_forward_logits_int8_kv(gpu_lib, oracle_built, name):
    shape, dl = SHAPES_KV[name]
    pair = make_pair(shape, dl, seed=13, kv_mode=2, max_prompt_len=40)
    toks = make_prompts(1, 33, shape.vocab, seed=14)[0]
    for role, om in ((sd.TARGET, pair.target), (sd.DRAFT, pair.draft)):
        g = pair.engine.forward_logits(role, toks)
        o = om.forward(toks, kv_mode=2)
        assert rel_err(g, o) < FP32_REL, (name, role, rel_err(g, o))


@pytest.mark.parametrize("name", list(SHAPES_KV))
@pytest.mark.parametrize("T", [0.0, 1.0])
def test_spec_int8_kv(gpu_lib, oracle_built, name, T):
    shape, dl = SHAPES_KV[name]
    pair = make_pair(shape, dl, seed=15, int8=True, kv_mode=2, max_batch=4, max_prompt_len=40)
    _, tg, sg, to, so, mg = run_both(pair, 3, 12, 40, 4, T, seed=31, use_uniforms=T > 0)
    exact, ties = compare_tokens(tg, to, mg, 12, greedy=T <= 0)
    assert exact + ties == 3 and ties <= 1


# Tensor-core GEMM path (bf16 activations, int8 weights, >= 64 rows): long
# prefills, and a vocabulary / width that are not multiples of the 256 x 64
# tile (column and K tails).
GEMM_SHAPES = {
    "cfg1": SHAPES["cfg1"],
    "ragged": (ModelShape(vocab=1000, d_model=192, n_heads=3, d_ff=320, n_layers=2, max_seq_len=200), 1),
}


@pytest.mark.parametrize("name", list(GEMM_SHAPES))
@pytest.mark.parametrize("kv_mode", [0, 1])
def test_forward_logits_bf16_gemm(gpu_lib, oracle_built, name, kv_mode):
    shape, dl = GEMM_SHAPES[name]
    pair = make_pair(shape, dl, seed=21, int8=True, act_bf16=True, kv_mode=kv_mode, max_prompt_len=160)
    toks = make_prompts(1, 150, shape.vocab, seed=22)[0]
    for role, om in ((sd.TARGET, pair.target), (sd.DRAFT, pair.draft)):
        g = pair.engine.forward_logits(role, toks)
        o = om.forward(toks, act_bf16=True, kv_mode=kv_mode)
        assert rel_err(g, o) < BF16_REL, (name, role, rel_err(g, o))


def test_greedy_spec_bf16_gemm(gpu_lib, oracle_built):
    # 16 requests x (k + 1) = 80 verify rows and 16 x 80 prefill rows take the GEMM
    shape, dl = GEMM_SHAPES["ragged"]
    pair = make_pair(shape, dl, seed=23, int8=True, act_bf16=True, kv_mode=1, max_batch=16, max_prompt_len=80)
    _, tg, sg, to, so, mg = run_both(pair, 16, 80, 24, 4, 0.0)
    exact, ties = compare_tokens(tg, to, mg, 80, greedy=True, tol=BF16_GREEDY_GAP)
    assert exact + ties == 16 and ties <= 4


def test_gemm_split_k_matches_unsplit(gpu_lib, oracle_built, monkeypatch):
    # few tiles over a long K: the residual GEMMs split K over clusters of up
    # to 8 CTAs; against the same engine built with splitting off, and the oracle
    shape = ModelShape(vocab=512, d_model=256, n_heads=4, d_ff=2048, n_layers=2, max_seq_len=200)
    toks = make_prompts(1, 150, shape.vocab, seed=31)[0]
    split = make_pair(shape, 1, seed=30, int8=True, act_bf16=True, kv_mode=1, max_prompt_len=160)
    monkeypatch.setenv("SPECDEC_GEMM_MAX_SPLIT", "1")
    whole = make_pair(shape, 1, seed=30, int8=True, act_bf16=True, kv_mode=1, max_prompt_len=160)
    a = split.engine.forward_logits(sd.TARGET, toks)
    b = whole.engine.forward_logits(sd.TARGET, toks)
    o = split.target.forward(toks, act_bf16=True, kv_mode=1)
    assert rel_err(a, b) < BF16_REL and rel_err(a, o) < BF16_REL and rel_err(b, o) < BF16_REL
    split.engine.close()
    whole.engine.close()


# Token trees (tree.cuh) against the oracle's path-by-path restatement
# (oracle/specdec_oracle.cpp: tree_one): greedy and both uniform sources.
def _tree_pair(name, seed, **kw):
    shape, dl = SHAPES[name]
    return make_pair(shape, dl, seed=seed, max_batch=4, max_prompt_len=40, **kw)


def _tree_both(pair, B, S, max_new, br, T, seed=9, use_uniforms=False, top_k=0, top_p=1.0):
    prompts = make_prompts(B, S, pair.shape.vocab, seed=4)
    uni = sd.philox_uniforms(seed, B, max_new + 2, oracle.tree_slots(br)) if use_uniforms else None
    tg, sg = pair.engine.generate_tree(prompts, max_new, br, T, top_k, top_p, seed, uniforms=uni)
    to, so, mg = oracle.oracle_generate_tree(pair.target, pair.draft, prompts, max_new, br, T, top_k, top_p, seed,
                                             uniforms=uni, act_bf16=pair.act_bf16, kv_mode=pair.kv_mode,
                                             cache_cap=pair.shape.max_seq_len)
    return tg, sg, to, so, mg


@pytest.mark.parametrize("name", ["small", "cfg1"])
@pytest.mark.parametrize("br", [(4, 3, 2, 1), (2, 2), (1, 1, 1, 1)])
def test_tree_greedy(gpu_lib, name, br):
    pair = _tree_pair(name, 41, max_tree_nodes=64)
    tg, sg, to, so, mg = _tree_both(pair, 3, 10, 30, list(br), 0.0)
    exact, ties = compare_tokens(tg, to, mg, 10, greedy=True)
    assert exact + ties == 3 and ties <= 1
    if ties == 0:
        assert np.array_equal(sg, so)


@pytest.mark.parametrize("name", ["small", "cfg1"])
@pytest.mark.parametrize("use_uniforms", [False, True])
def test_tree_sampled(gpu_lib, name, use_uniforms):
    pair = _tree_pair(name, 42, max_tree_nodes=64)
    tg, sg, to, so, mg = _tree_both(pair, 3, 10, 30, [4, 3, 2, 1], 1.0, use_uniforms=use_uniforms)
    exact, ties = compare_tokens(tg, to, mg, 10, greedy=False)
    assert exact + ties == 3 and ties <= 1


def test_tree_int8_kv_and_weights(gpu_lib):
    pair = _tree_pair("cfg1", 43, max_tree_nodes=64, int8=True, kv_mode=2)
    tg, sg, to, so, mg = _tree_both(pair, 2, 10, 24, [3, 2, 1], 1.0, use_uniforms=True)
    exact, ties = compare_tokens(tg, to, mg, 10, greedy=False)
    assert exact + ties == 2 and ties <= 1


def test_tree_chain_equivalence_gpu(gpu_lib):
    # a 1/1/1/1 tree is the k = 4 chain (greedy, consistent catch-up)
    pair = _tree_pair("cfg1", 44, max_tree_nodes=64)
    prompts = make_prompts(3, 12, pair.shape.vocab, seed=5)
    tt, st = pair.engine.generate_tree(prompts, 40, [1, 1, 1, 1], 0.0)
    tc, sc = pair.engine.generate_speculative(prompts, 40, 4, 0.0, draft_catchup=sd.CATCHUP_CORRECT)
    assert np.array_equal(tt, tc)


# Grouped-query and multi-query attention (MultiHeadAttention's num_kv_heads,
# src/nn/layer.cpp:471-489, 565-591; the reference's TransformerDecoder always
# builds full multi-head attention, so these compare with the restatement).
@pytest.mark.parametrize("kv_heads", [2, 1])
@pytest.mark.parametrize("kv_mode", [0, 2])
def test_gqa_forward_and_greedy_spec(gpu_lib, oracle_built, kv_heads, kv_mode):
    shape = ModelShape(vocab=512, d_model=128, n_heads=4, d_ff=256, n_layers=2, max_seq_len=160, n_kv_heads=kv_heads)
    pair = make_pair(shape, 1, seed=40 + kv_heads, kv_mode=kv_mode, max_prompt_len=40)
    toks = make_prompts(1, 33, shape.vocab, seed=41)[0]
    for role, om in ((sd.TARGET, pair.target), (sd.DRAFT, pair.draft)):
        g = pair.engine.forward_logits(role, toks)
        o = om.forward(toks, kv_mode=kv_mode)
        assert rel_err(g, o) < FP32_REL, (role, rel_err(g, o))
    _, tg, sg, to, so, mg = run_both(pair, 3, 12, 30, 4, 0.0)
    exact, ties = compare_tokens(tg, to, mg, 12, greedy=True)
    assert exact + ties == 3 and ties <= 1


# Large vocabularies: the draft sampler splits each request's row over a
# cluster of CTAs (no top-k / top-p); odd and power-of-two vocabularies.
@pytest.mark.parametrize("vocab", [9001, 16384])
@pytest.mark.parametrize("T,uniforms", [(0.0, False), (1.0, False), (0.8, True)])
def test_spec_large_vocab_cluster_sampler(gpu_lib, oracle_built, monkeypatch, vocab, T, uniforms):
    shape = ModelShape(vocab=vocab, d_model=64, n_heads=4, d_ff=128, n_layers=2, max_seq_len=96)
    pair = make_pair(shape, 1, seed=50, max_batch=4, max_prompt_len=16)
    _, tg, sg, to, so, mg = run_both(pair, 4, 9, 40, 4, T, seed=17, use_uniforms=uniforms)
    exact, ties = compare_tokens(tg, to, mg, 9, greedy=T <= 0)
    assert exact + ties == 4 and ties <= 1
    # the same engine with one CTA per request
    monkeypatch.setenv("SPECDEC_SAMPLE_MAX_CLUSTER", "1")
    one = make_pair(shape, 1, seed=50, max_batch=4, max_prompt_len=16)
    _, t1, s1, _, _, _ = run_both(one, 4, 9, 40, 4, T, seed=17, use_uniforms=uniforms)
    for b in range(4):
        d = np.nonzero(t1[b] != tg[b])[0]
        if d.size:  # only at an oracle near-tie
            assert mg[b, : int(d[0]) - 9 + 1].min() < (1e-4 if T <= 0 else 2e-5)
    pair.engine.close()
    one.engine.close()


# Tensor-core attention (attn_tc.cuh: bf16 caches, head_dim 64, groups of 16
# or more queries): prefill chunks and token-tree verify blocks, against the
# CUDA-core attention kernel and the oracle.
def test_attention_tc_prefill_matches_cuda_core(gpu_lib, oracle_built, monkeypatch):
    shape = ModelShape(vocab=1000, d_model=256, n_heads=4, d_ff=512, n_layers=2, max_seq_len=400)
    toks = make_prompts(1, 300, shape.vocab, seed=61)[0]  # 3 query tiles, 3 cache tiles
    tc = make_pair(shape, 1, seed=60, int8=True, act_bf16=True, kv_mode=1, max_prompt_len=320)
    monkeypatch.setenv("SPECDEC_ATTN_TC", "0")
    cc = make_pair(shape, 1, seed=60, int8=True, act_bf16=True, kv_mode=1, max_prompt_len=320)
    a = tc.engine.forward_logits(sd.TARGET, toks)
    b = cc.engine.forward_logits(sd.TARGET, toks)
    o = tc.target.forward(toks, act_bf16=True, kv_mode=1)
    assert rel_err(a, b) < BF16_REL and rel_err(a, o) < BF16_REL, (rel_err(a, b), rel_err(a, o))
    tc.engine.close()
    cc.engine.close()


@pytest.mark.parametrize("br", [(4, 3, 2, 1), (2, 2, 2, 2)])
def test_tree_greedy_bf16_tensor_core_attention(gpu_lib, oracle_built, br):
    shape, dl = SHAPES["cfg1"]
    pair = make_pair(shape, dl, seed=62, int8=True, act_bf16=True, kv_mode=1, max_batch=4, max_prompt_len=40,
                     max_tree_nodes=64)
    tg, sg, to, so, mg = _tree_both(pair, 3, 20, 30, list(br), 0.0)
    exact, ties = compare_tokens(tg, to, mg, 20, greedy=True, tol=BF16_GREEDY_GAP)
    assert exact + ties == 3
