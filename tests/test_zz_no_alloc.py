"""The no-allocation forward (specdec_forward_logits_noalloc).

It exists for callers that must not allocate device memory when they run a
forward pass (a host runtime that owns all device memory, or a loop where an
allocation could stall the GPU): they pass device buffers they already own,
and the library works out of one fixed device array.  Each case calls it
twice in a row (the calls share the array) and checks the logits against
specdec_forward_logits and against the CPU oracle, and the device status word
it writes.  This file runs last so that a failure here never hides another
test's result; it must also pass on its own in a fresh process.
"""
import numpy as np
import pytest

import specdec_b200 as sd
from helpers import make_pair
from specdec_b200.synth import ModelShape, make_params, make_prompts

pytestmark = pytest.mark.gpu

FP32_REL = 1e-3
BF16_REL = 2e-2

CFG1 = ModelShape(vocab=2048, d_model=256, n_heads=4, d_ff=1024, n_layers=4, max_seq_len=128)


def _rel(a, b):
    return float(np.max(np.abs(a - b)) / max(1e-30, float(np.max(np.abs(b)))))


# (int8 weights, bf16 activations, kv mode, sequence lengths, caller stream):
# fp32 GEMV paths; the bf16 tensor-core GEMM with LayerNorm rows staged in
# the scratch array (64 rows and more) over a bf16 cache; the int8 cache with
# its staged rows and scale planes in the scratch array
CASES = [
    (False, False, 0, (40, 17), False),
    (True, False, 0, (40, 17), True),
    (True, True, 1, (96, 70), True),
    (True, True, 2, (80, 33), False),
]


@pytest.mark.parametrize("int8,bf16,kv,lens,own_stream", CASES)
def test_noalloc_forward_matches(gpu_lib, oracle_built, int8, bf16, kv, lens, own_stream):
    import torch

    pair = make_pair(CFG1, 1, seed=12, int8=int8, act_bf16=bf16, kv_mode=kv, max_prompt_len=128)
    eng = pair.engine
    tol = BF16_REL if bf16 else FP32_REL
    stream = torch.cuda.Stream() if own_stream else None
    status = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    for role, om in ((sd.TARGET, pair.target), (sd.DRAFT, pair.draft)):
        for call, S in enumerate(lens):  # two calls in a row share the scratch array
            toks = make_prompts(1, S, CFG1.vocab, seed=30 + call)[0]
            want = eng.forward_logits(role, toks)
            ref = om.forward(toks, act_bf16=bf16, kv_mode=kv)
            d_tok = torch.from_numpy(toks.astype(np.int32)).cuda()
            d_log = torch.full((S, CFG1.vocab), float("nan"), dtype=torch.float32, device="cuda")
            status.fill_(-1)
            torch.cuda.synchronize()
            eng.forward_logits_noalloc(role, d_tok.data_ptr(), S, d_log.data_ptr(),
                                       stream.cuda_stream if stream is not None else 0, status.data_ptr())
            torch.cuda.synchronize()
            got = d_log.cpu().numpy()
            assert int(status.item()) == 0
            assert np.isfinite(got).all()
            assert _rel(got, want) < tol, (role, call, _rel(got, want))
            assert _rel(got, ref) < tol, (role, call, _rel(got, ref))
    eng.close()


def test_noalloc_rejects_oversized_work(gpu_lib):
    import torch

    shape = ModelShape(vocab=512, d_model=1024, n_heads=8, d_ff=4096, n_layers=8, max_seq_len=1024)
    eng = sd.Engine(shape, draft_layers=1, max_batch=1, max_prompt_len=8)
    eng.load_params(sd.TARGET, make_params(shape, seed=1))
    S = 1000
    d_tok = torch.zeros(S, dtype=torch.int32, device="cuda")
    d_log = torch.zeros((S, shape.vocab), dtype=torch.float32, device="cuda")
    with pytest.raises(sd.SpecDecError) as e:
        eng.forward_logits_noalloc(sd.TARGET, d_tok.data_ptr(), S, d_log.data_ptr(), 0)
    assert e.value.code == 1 and "scratch" in str(e.value)
    eng.close()


def test_noalloc_respects_each_models_max_seq(gpu_lib):
    """A draft with a shorter max_seq_len than the target's: the draft's own
    capacity bounds the sequence (the reference throws past max_seq_len)."""
    import torch

    target = ModelShape(vocab=256, d_model=64, n_heads=4, d_ff=128, n_layers=2, max_seq_len=96)
    draft = ModelShape(vocab=256, d_model=64, n_heads=4, d_ff=128, n_layers=1, max_seq_len=32)
    eng = sd.Engine(target, draft=draft, max_batch=1, max_prompt_len=16)
    P = make_params(target, seed=2)
    eng.load_params(sd.TARGET, P)
    eng.load_params(sd.DRAFT, make_params(draft, seed=3))
    S = 48
    d_tok = torch.zeros(S, dtype=torch.int32, device="cuda")
    d_log = torch.zeros((S, target.vocab), dtype=torch.float32, device="cuda")
    eng.forward_logits_noalloc(sd.TARGET, d_tok.data_ptr(), S, d_log.data_ptr(), 0)
    torch.cuda.synchronize()
    with pytest.raises(sd.SpecDecError) as e:
        eng.forward_logits_noalloc(sd.DRAFT, d_tok.data_ptr(), S, d_log.data_ptr(), 0)
    assert e.value.code == 4
    eng.close()
