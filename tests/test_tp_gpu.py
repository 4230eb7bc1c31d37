"""Tensor parallelism (specdec_create_tp) on two GPUs against the CPU oracle:
each rank holds half of the heads and FFN columns and the two partial
projections meet in an NCCL all-reduce; rank 0's logits and tokens must match
the single-model oracle like the one-GPU path does.  Skipped with fewer than
two GPUs."""
import multiprocessing as mp
import os
import queue

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

WORLD = 2


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def cfg_uid2(rank, idq):
    """A second NCCL id for a second communicator, passed like the first."""
    import specdec_b200 as sd
    if rank == 0:
        uid = sd.tp_unique_id()
        for _ in range(WORLD - 1):
            idq.put(uid)
        return uid
    return idq.get(timeout=120)


def _worker(rank, idq, cfg, q):
    try:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        import sys
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, os.path.join(root, "neural-network_b200"))
        import specdec_b200 as sd
        # rank 0 makes the NCCL id with the same NCCL copy both ranks load
        if rank == 0:
            uid = sd.tp_unique_id()
            for _ in range(WORLD - 1):
                idq.put(uid)
        else:
            uid = idq.get(timeout=120)
        from specdec_b200.synth import ModelShape, draft_params, make_params, make_prompts
        shape = ModelShape(**cfg["shape"])
        P = make_params(shape, seed=cfg["seed"], bias_std=0.02, ln_jitter=0.05)
        eng = sd.Engine(shape, draft_layers=1, weight_dtype=cfg["wdt"], act_dtype=cfg["adt"], kv_dtype=cfg["kvdt"],
                        max_batch=3, max_lookahead=4, max_prompt_len=cfg["S"], device=rank,
                        tp_rank=rank, tp_world=WORLD, tp_id=uid)
        eng.load_params(sd.TARGET, P)
        toks = make_prompts(1, cfg["S"], shape.vocab, seed=9)[0]
        lg = eng.forward_logits(sd.TARGET, toks)
        prompts = make_prompts(3, 12, shape.vocab, seed=1)
        tg, _ = eng.generate_speculative(prompts, 24, 4, 0.0)
        uni = sd.philox_uniforms(77, 3, 26, 9)
        ts, _ = eng.generate_speculative(prompts, 24, 4, 1.0, seed=77, uniforms=uni)
        eng.close()
        # the round-level session on a handle loaded from device arrays (each
        # rank slices and quantises its part on its GPU): the same tokens
        import torch
        eng = sd.Engine(shape, draft_layers=1, weight_dtype=cfg["wdt"], act_dtype=cfg["adt"], kv_dtype=cfg["kvdt"],
                        max_batch=3, max_lookahead=4, max_prompt_len=cfg["S"], device=rank,
                        tp_rank=rank, tp_world=WORLD, tp_id=cfg_uid2(rank, idq))
        eng.load_params_device(sd.TARGET, [torch.from_numpy(np.ascontiguousarray(p, np.float32)).to(f"cuda:{rank}")
                                           for p in P])
        eng.prefill(prompts, 24, 4, 1.0, seed=77, uniforms=uni)
        got = np.zeros(3, np.int64)
        for _ in range(24):
            _, cnt = eng.step(1)
            got += cnt
            if np.all(got >= 23):  # the first of the 24 new tokens came from the prefill
                break
        full, _ = eng.session_tokens()
        eng.close()
        if rank == 0:
            q.put(("ok", lg, tg, ts, full))
    except Exception as e:  # report instead of hanging the parent
        q.put(("err", f"rank {rank}: {e!r}"))


def _run(cfg):
    ctx = mp.get_context("spawn")
    q, idq = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, idq, cfg, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    try:
        res = q.get(timeout=240)
    except queue.Empty:
        res = ("err", "timeout")
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[0] == "ok", res[1]
    return res[1:]


@pytest.mark.skipif(_gpus() < WORLD, reason="needs two GPUs")
@pytest.mark.parametrize("mode", ["fp32", "bf16_int8"])
def test_tensor_parallel_matches_oracle(oracle_built, mode):
    import oracle
    import specdec_b200 as sd
    from helpers import BF16_GREEDY_GAP, compare_tokens
    from specdec_b200.synth import ModelShape, draft_params, make_params, make_prompts

    shp = dict(vocab=2048, d_model=256, n_heads=4, d_ff=1024, n_layers=2, max_seq_len=200)
    bf = mode != "fp32"
    cfg = {"shape": shp, "seed": 3, "S": 80 if bf else 33, "wdt": sd.INT8 if bf else sd.F32,
           "adt": sd.BF16 if bf else sd.F32, "kvdt": sd.BF16 if bf else sd.F32}
    lg, tg, ts, session = _run(cfg)
    assert np.array_equal(session, ts)
    shape = ModelShape(**shp)
    P = make_params(shape, seed=3, bias_std=0.02, ln_jitter=0.05)
    t = oracle.Oracle(shape, P, int8=bf)
    d = oracle.Oracle(shape.with_layers(1), draft_params(shape, P, 1), int8=bf)
    toks = make_prompts(1, cfg["S"], shape.vocab, seed=9)[0]
    o = t.forward(toks, act_bf16=bf, kv_mode=1 if bf else 0)
    rel = float(np.max(np.abs(lg - o)) / np.max(np.abs(o)))
    assert rel < (2e-2 if bf else 1e-3), rel
    prompts = make_prompts(3, 12, shape.vocab, seed=1)
    to, _, mg = oracle.oracle_generate_speculative(t, d, prompts, 24, 4, 0.0, act_bf16=bf, kv_mode=1 if bf else 0,
                                                   cache_cap=200)
    ex, ti = compare_tokens(tg, to, mg, 12, greedy=True, tol=BF16_GREEDY_GAP if bf else None)
    assert ex + ti == 3
    if not bf:
        uni = sd.philox_uniforms(77, 3, 26, 9)
        to, _, mg = oracle.oracle_generate_speculative(t, d, prompts, 24, 4, 1.0, seed=77, uniforms=uni,
                                                       cache_cap=200)
        ex, ti = compare_tokens(ts, to, mg, 12, greedy=False)
        assert ex + ti == 3 and ti <= 1
