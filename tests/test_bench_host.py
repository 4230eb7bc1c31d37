"""Host-side pieces of bench.py, on the CPU: the algorithmic bytes per round
that the round roofline divides by, and the GPU weight synthesis of the large
workload (run here on a CPU device at a small shape)."""
import importlib.util
import os

import numpy as np

from specdec_b200.synth import ModelShape, param_kinds, param_shapes, workload

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_round_bytes_of_the_large_workload():
    b = _bench()
    wl = workload("large")
    ab = b.algorithmic_bytes_per_round(wl, True, 2048 + 256)
    d, F, V = 4096, 11008, 32000
    per_layer = 4 * d * d + 3 * d * F  # int8 q, k, v, o and SwiGLU gate, up, down
    assert ab["w_target"] == 32 * per_layer + d * V  # 6.6 G weights plus the lm_head
    assert ab["w_draft"] == 4 * per_layer + d * V
    assert ab["weights"] == 4 * ab["w_draft"] + ab["w_target"]
    # bf16 K and V rows of 4096 values per position and layer
    kv_tok_layer = 2 * d * 2
    B, k = wl.batch, wl.lookahead
    kv = B * 2304 * kv_tok_layer * (k * 4 + 32) + B * kv_tok_layer * ((k + 1) * 4 + (k + 1) * 32)
    assert ab["kv"] == kv


def test_device_params_shapes_and_distributions():
    import torch

    b = _bench()
    shape = ModelShape(vocab=300, d_model=64, n_heads=4, d_ff=128, n_layers=2, max_seq_len=16)
    P = b.device_params(shape, 0, torch.device("cpu"))
    assert [p.shape for p in P] == [tuple(s) for s in param_shapes(shape)]
    for p, kind in zip(P, param_kinds(shape)):
        assert p.dtype == np.float32
        if kind == "w":
            assert abs(float(p.std()) - 0.02) < 0.004
        elif kind == "head_w":
            assert abs(float(p.std()) - 4.0 / np.sqrt(64)) < 0.05
        elif kind == "g":
            assert np.all(p == 1.0)
        elif kind in ("b", "beta", "head_b"):
            assert np.all(p == 0.0)
    # seeded: the same seed gives the same weights
    Q = b.device_params(shape, 0, torch.device("cpu"))
    assert all(np.array_equal(x, y) for x, y in zip(P, Q))
