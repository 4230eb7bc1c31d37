"""Weight files: the reference's NETW v1 parameter format
(serialization::save_parameters / load_parameters,
src/core/serialization.cpp:8-107, reached through Layer::save_weights /
load_weights, src/nn/layer.cpp:463-469) and specdec_load_netw, which reads it
into the B200 engine.  The fixtures tests/golden/*_target.netw were written by
the unmodified reference (tests/golden/make_golden.py)."""
import os
import struct

import numpy as np
import pytest

import oracle
import specdec_b200 as sd
from specdec_b200.synth import ModelShape, make_params

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# name -> (shape, weight seed, bias / LayerNorm jitter), as make_golden.py
NETW = {
    "tiny8": (ModelShape(vocab=8, d_model=8, n_heads=2, d_ff=16, n_layers=2, max_seq_len=64), 11, 0.05),
    "small": (ModelShape(vocab=97, d_model=32, n_heads=4, d_ff=64, n_layers=2, max_seq_len=160), 13, 0.02),
}


def read_netw(path):
    """The file as a list of (shape, float32 array)."""
    with open(path, "rb") as f:
        raw = f.read()
    assert raw[:4] == b"NETW"
    version, count = struct.unpack_from("<HI", raw, 4)
    assert version == 1
    off = 10
    out = []
    for _ in range(count):
        (dims,) = struct.unpack_from("<I", raw, off)
        off += 4
        shape = struct.unpack_from(f"<{dims}Q", raw, off)
        off += 8 * dims
        (n,) = struct.unpack_from("<Q", raw, off)
        off += 8
        out.append((tuple(shape), np.frombuffer(raw, np.float32, n, off).copy()))
        off += 4 * n
    assert off == len(raw)
    return out


def write_netw(path, tensors, magic=b"NETW", version=1):
    with open(path, "wb") as f:
        f.write(magic)
        f.write(struct.pack("<HI", version, len(tensors)))
        for shape, data in tensors:
            f.write(struct.pack("<I", len(shape)))
            f.write(struct.pack(f"<{len(shape)}Q", *shape))
            f.write(struct.pack("<Q", data.size))
            f.write(np.ascontiguousarray(data, np.float32).tobytes())


@pytest.mark.parametrize("name", list(NETW))
def test_reference_netw_fixture_holds_the_injected_weights(name):
    shape, seed, jit = NETW[name]
    P = make_params(shape, seed=seed, bias_std=jit, ln_jitter=jit)
    ts = read_netw(os.path.join(GOLDEN_DIR, f"{name}_target.netw"))
    assert len(ts) == len(P)
    d, F, V = shape.d_model, shape.d_ff, shape.vocab
    assert ts[0][0] == (V, d)           # Embedding [V, d]
    assert ts[1][0] == (d, d)           # q weight [in, out]
    assert ts[2][0] == (1, d)           # q bias [1, out]
    assert ts[9][0] == (d, F)           # SwiGLU gate weight
    assert ts[13][0] == (F, d)          # down weight
    assert ts[15][0] == (d,)            # LayerNorm gamma
    assert ts[-2][0] == (d, V) and ts[-1][0] == (1, V)
    for (s, a), p in zip(ts, P):
        assert np.array_equal(a, np.ascontiguousarray(p, np.float32).ravel())


@pytest.mark.parametrize("name", list(NETW))
def test_reference_reads_its_own_fixture(oracle_built, golden, name):
    if not oracle.reference_available():
        pytest.skip("reference library not built here")
    shape, seed, jit = NETW[name]
    m = oracle.Reference(shape, [np.zeros(np.shape(p), np.float32) for p in make_params(shape, seed=seed)],
                         requires_grad=False)
    m.load_weights(os.path.join(GOLDEN_DIR, f"{name}_target.netw"))
    got = m.forward(golden[f"{name}/prompt"])
    ref = golden[f"{name}/logits_target"]
    assert np.max(np.abs(got - ref)) <= 1e-5 * max(1.0, float(np.max(np.abs(ref))))


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(NETW))
@pytest.mark.parametrize("int8", [False, True])
def test_engine_loads_reference_netw(gpu_lib, oracle_built, golden, name, int8):
    shape, seed, jit = NETW[name]
    P = make_params(shape, seed=seed, bias_std=jit, ln_jitter=jit)
    a = sd.Engine(shape, draft_layers=1, weight_dtype=sd.INT8 if int8 else sd.F32, max_batch=1, max_prompt_len=16)
    a.load_weights(sd.TARGET, os.path.join(GOLDEN_DIR, f"{name}_target.netw"))
    b = sd.Engine(shape, draft_layers=1, weight_dtype=sd.INT8 if int8 else sd.F32, max_batch=1, max_prompt_len=16)
    b.load_params(sd.TARGET, P)
    prompt = golden[f"{name}/prompt"]
    la, lb = a.forward_logits(sd.TARGET, prompt), b.forward_logits(sd.TARGET, prompt)
    assert np.array_equal(la, lb)  # the same weights on the device
    if not int8:
        ref = golden[f"{name}/logits_target"]
        assert np.max(np.abs(la - ref)) / np.max(np.abs(ref)) < 1e-3
    # the draft (the target's first layer + shared head) came with the file
    assert np.array_equal(a.forward_logits(sd.DRAFT, prompt), b.forward_logits(sd.DRAFT, prompt))
    a.close()
    b.close()


@pytest.mark.gpu
def test_engine_netw_errors(gpu_lib, tmp_path):
    # each failure of serialization::load_parameters, with its message
    shape, seed, jit = NETW["tiny8"]
    ts = read_netw(os.path.join(GOLDEN_DIR, "tiny8_target.netw"))
    eng = sd.Engine(shape, draft_layers=1, max_batch=1, max_prompt_len=8)

    def expect(path, text):
        with pytest.raises(sd.SpecDecError) as e:
            eng.load_weights(sd.TARGET, str(path))
        assert e.value.code == 1 and text in str(e.value), str(e.value)

    expect(tmp_path / "missing.netw", "Failed to open file for reading")
    write_netw(tmp_path / "magic.netw", ts, magic=b"NETX")
    expect(tmp_path / "magic.netw", "Invalid file format signature.")
    write_netw(tmp_path / "ver.netw", ts, version=2)
    expect(tmp_path / "ver.netw", "Unsupported serialization file version: 2")
    write_netw(tmp_path / "count.netw", ts[:-1])
    expect(tmp_path / "count.netw", f"Tensor count mismatch (file has {len(ts) - 1}, model has {len(ts)}).")
    bad = list(ts)
    bad[2] = ((shape.d_model,), bad[2][1])
    write_netw(tmp_path / "rank.netw", bad)
    expect(tmp_path / "rank.netw", "Tensor dimension count mismatch.")
    bad = list(ts)
    bad[0] = ((shape.vocab + 1, shape.d_model), np.zeros((shape.vocab + 1) * shape.d_model, np.float32))
    write_netw(tmp_path / "shape.netw", bad)
    expect(tmp_path / "shape.netw", "Tensor shape mismatch at dimension 0")
    bad = list(ts)
    bad[3] = (bad[3][0], bad[3][1][:-1])
    write_netw(tmp_path / "numel.netw", bad)
    expect(tmp_path / "numel.netw", "Tensor element count mismatch.")
    raw = open(os.path.join(GOLDEN_DIR, "tiny8_target.netw"), "rb").read()
    (tmp_path / "cut.netw").write_bytes(raw[:-12])
    expect(tmp_path / "cut.netw", "truncated")
    # still usable: the good file loads
    eng.load_weights(sd.TARGET, os.path.join(GOLDEN_DIR, "tiny8_target.netw"))
    eng.close()
