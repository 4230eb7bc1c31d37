"""The no-allocation forward (specdec_forward_logits_noalloc).

It exists for callers that must not allocate device memory when they run a
forward pass (a host runtime that owns all device memory, or a loop where an
allocation could stall the GPU): they pass device buffers they already own,
and the library works out of one fixed device array.  This file runs last so
that a failure here never hides another test's result; it must also pass on
its own in a fresh process.
"""
import numpy as np
import pytest

import specdec_b200 as sd
from helpers import make_pair
from specdec_b200.synth import ModelShape, make_prompts

pytestmark = pytest.mark.gpu

FP32_REL = 1e-3


def _rel(a, b):
    return float(np.max(np.abs(a - b)) / max(1e-30, float(np.max(np.abs(b)))))


@pytest.mark.parametrize("int8", [False, True])
def test_noalloc_forward_matches_forward_logits(gpu_lib, oracle_built, int8):
    import torch

    shape = ModelShape(vocab=2048, d_model=256, n_heads=4, d_ff=1024, n_layers=4, max_seq_len=128)
    pair = make_pair(shape, 1, seed=12, int8=int8, max_prompt_len=64)
    eng = pair.engine
    for role in (sd.TARGET, sd.DRAFT):
        for call, S in enumerate((40, 17)):  # two calls in a row share the scratch array
            toks = make_prompts(1, S, shape.vocab, seed=30 + call)[0]
            want = eng.forward_logits(role, toks)
            d_tok = torch.from_numpy(toks.astype(np.int32)).cuda()
            d_log = torch.full((S, shape.vocab), float("nan"), dtype=torch.float32, device="cuda")
            torch.cuda.synchronize()
            eng.forward_logits_noalloc(role, d_tok.data_ptr(), S, d_log.data_ptr(), 0)
            torch.cuda.synchronize()
            got = d_log.cpu().numpy()
            assert np.isfinite(got).all()
            assert _rel(got, want) < FP32_REL, (role, call, _rel(got, want))


def test_noalloc_rejects_oversized_work(gpu_lib):
    import torch

    shape = ModelShape(vocab=512, d_model=1024, n_heads=8, d_ff=4096, n_layers=8, max_seq_len=1024)
    eng = sd.Engine(shape, draft_layers=1, max_batch=1, max_prompt_len=8)
    from specdec_b200.synth import make_params
    eng.load_params(sd.TARGET, make_params(shape, seed=1))
    S = 1000
    d_tok = torch.zeros(S, dtype=torch.int32, device="cuda")
    d_log = torch.zeros((S, shape.vocab), dtype=torch.float32, device="cuda")
    with pytest.raises(sd.SpecDecError) as e:
        eng.forward_logits_noalloc(sd.TARGET, d_tok.data_ptr(), S, d_log.data_ptr(), 0)
    assert e.value.code == 1 and "scratch" in str(e.value)
    eng.close()
