"""Seeded synthetic inputs for the speculative-decoding path.

The reference publishes no checkpoints or datasets for this path; every
benchmark and parity case runs on seeded random weights and uniform-random
prompt tokens.  Everything here is plain numpy so the same arrays feed the
B200 engine, the CPU restatement and the reference library.

Parameter order follows ``TransformerDecoder::parameters()``
(src/nn/layer.cpp:1140-1154): the token embedding, then per layer the attention
projections q, k, v, out (weight, bias each; src/nn/layer.cpp:491-502), the
SwiGLU gate, up, down (src/nn/layer.cpp:1712-1721), LayerNorm 1 and 2
(gamma, beta; src/nn/layer.cpp:1079-1090), and finally the lm_head weight and
bias.  Dense weights are stored ``[in, out]`` row-major as in
src/nn/layer.cpp:153.

The ``cfg`` architecture (pre-LN, GELU FFN, learned positions, final LN) has
no reference counterpart; its order is: embedding, positions, per layer
[ln1 g/b, q, k, v, o, ln2 g/b, fc1, fc2], final LN g/b, lm_head.
"""
from __future__ import annotations

from dataclasses import dataclass, field, replace
from typing import List, Tuple

import numpy as np

ARCH_REF = 0
ARCH_CFG = 1


@dataclass(frozen=True)
class ModelShape:
    vocab: int
    d_model: int
    n_heads: int
    d_ff: int
    n_layers: int
    max_seq_len: int
    n_kv_heads: int = 0          # 0 -> n_heads (the reference's default, layer.cpp:474)
    arch: int = ARCH_REF

    @property
    def kv_heads(self) -> int:
        return self.n_kv_heads or self.n_heads

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads

    def with_layers(self, n: int) -> "ModelShape":
        return replace(self, n_layers=n)


def param_shapes(m: ModelShape) -> List[Tuple[int, ...]]:
    d, F, V = m.d_model, m.d_ff, m.vocab
    kvd = m.kv_heads * m.head_dim
    out: List[Tuple[int, ...]] = [(V, d)]
    if m.arch == ARCH_CFG:
        out.append((m.max_seq_len, d))
    for _ in range(m.n_layers):
        attn = [(d, d), (1, d), (d, kvd), (1, kvd), (d, kvd), (1, kvd), (d, d), (1, d)]
        if m.arch == ARCH_REF:
            out += attn
            out += [(d, F), (1, F), (d, F), (1, F), (F, d), (1, d)]
            out += [(d,), (d,), (d,), (d,)]
        else:
            out += [(d,), (d,)] + attn + [(d,), (d,)]
            out += [(d, F), (1, F), (F, d), (1, d)]
    if m.arch == ARCH_CFG:
        out += [(d,), (d,)]
    out += [(d, V), (1, V)]
    return out


def param_kinds(m: ModelShape) -> List[str]:
    """'emb' | 'pos' | 'w' | 'b' | 'g' (LN gamma) | 'beta' | 'head_w' | 'head_b'."""
    kinds = ["emb"]
    if m.arch == ARCH_CFG:
        kinds.append("pos")
    for _ in range(m.n_layers):
        attn = ["w", "b"] * 4
        if m.arch == ARCH_REF:
            kinds += attn + ["w", "b"] * 3 + ["g", "beta", "g", "beta"]
        else:
            kinds += ["g", "beta"] + attn + ["g", "beta"] + ["w", "b"] * 2
    if m.arch == ARCH_CFG:
        kinds += ["g", "beta"]
    kinds += ["head_w", "head_b"]
    return kinds


def params_per_layer(m: ModelShape) -> int:
    return 18 if m.arch == ARCH_REF else 16


def make_params(m: ModelShape, seed: int = 0, std: float = 0.02,
                head_std: float | None = None, bias_std: float = 0.0,
                ln_jitter: float = 0.0, emb_std: float | None = None) -> List[np.ndarray]:
    """Seeded N(0, std) weights.

    Biases are N(0, bias_std) (0 -> zeros), LayerNorm gamma = 1 + N(0, ln_jitter),
    beta = N(0, ln_jitter).  head_std defaults to 4/sqrt(d_model) so logits have
    a standard deviation near 4 after the unit-variance LayerNorm output.
    """
    rng = np.random.default_rng(seed)
    if head_std is None:
        head_std = 4.0 / np.sqrt(m.d_model)
    if emb_std is None:
        emb_std = std
    out: List[np.ndarray] = []
    for shape, kind in zip(param_shapes(m), param_kinds(m)):
        n = int(np.prod(shape))
        if kind == "emb" or kind == "pos":
            a = rng.standard_normal(n, dtype=np.float32) * np.float32(emb_std)
        elif kind == "w":
            a = rng.standard_normal(n, dtype=np.float32) * np.float32(std)
        elif kind == "head_w":
            a = rng.standard_normal(n, dtype=np.float32) * np.float32(head_std)
        elif kind in ("b", "head_b"):
            a = (rng.standard_normal(n, dtype=np.float32) * np.float32(bias_std)
                 if bias_std > 0 else np.zeros(n, np.float32))
        elif kind == "g":
            a = np.ones(n, np.float32)
            if ln_jitter > 0:
                a += rng.standard_normal(n, dtype=np.float32) * np.float32(ln_jitter)
        else:  # beta
            a = (rng.standard_normal(n, dtype=np.float32) * np.float32(ln_jitter)
                 if ln_jitter > 0 else np.zeros(n, np.float32))
        out.append(np.ascontiguousarray(a.reshape(shape), dtype=np.float32))
    return out


def device_params(m: ModelShape, seed: int, dev) -> List[np.ndarray]:
    """Seeded synthetic weights with make_params' distributions (N(0, 0.02)
    weights and embedding, N(0, 4/sqrt(d_model)) lm_head, zero biases, unit
    LayerNorm), drawn by torch on `dev` (a CUDA device: seconds for the large
    model's 6.9 G values, which numpy draws in minutes) and returned as host
    fp32 arrays.  The stream differs from make_params'; the benchmarks and
    profiling probes use it, the parity tests use make_params."""
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    out: List[np.ndarray] = []
    for shape, kind in zip(param_shapes(m), param_kinds(m)):
        n = int(np.prod(shape))
        if kind in ("emb", "pos", "w", "head_w"):
            std = 4.0 / np.sqrt(m.d_model) if kind == "head_w" else 0.02
            a = torch.empty(n, dtype=torch.float32, device=dev).normal_(0.0, std, generator=g).cpu().numpy()
        elif kind == "g":
            a = np.ones(n, np.float32)
        else:
            a = np.zeros(n, np.float32)
        out.append(a.reshape(shape))
    return out


def device_param_tensors(m: ModelShape, seed: int, dev) -> list:
    """device_params' weights as contiguous fp32 torch tensors left on `dev`
    (for Engine.load_params_device: no host copy of a multi-GB model)."""
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    out = []
    for shape, kind in zip(param_shapes(m), param_kinds(m)):
        n = int(np.prod(shape))
        if kind in ("emb", "pos", "w", "head_w"):
            std = 4.0 / np.sqrt(m.d_model) if kind == "head_w" else 0.02
            a = torch.empty(n, dtype=torch.float32, device=dev).normal_(0.0, std, generator=g)
        elif kind == "g":
            a = torch.ones(n, dtype=torch.float32, device=dev)
        else:
            a = torch.zeros(n, dtype=torch.float32, device=dev)
        out.append(a)
    return out


def draft_params(target: ModelShape, params: List[np.ndarray], n_draft_layers: int) -> List[np.ndarray]:
    """The draft used by every config: the target's first n layers + shared lm_head."""
    per = params_per_layer(target)
    head = 2
    lead = 1 if target.arch == ARCH_REF else 2
    body = params[lead: lead + per * n_draft_layers]
    tail = params[-head:] if target.arch == ARCH_REF else params[-4:]
    return list(params[:lead]) + list(body) + list(tail)


def make_prompts(B: int, S: int, vocab: int, seed: int = 1) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.integers(0, vocab, size=(B, S), dtype=np.int64)


# ---------------------------------------------------------------------------
# Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as easy
# as 1, 2, 3", SC'11), vectorised in numpy.  u[b][round][slot] uses key
# (seed & 0xffffffff, seed >> 32) and counter (slot // 4, round, b, 0x53504543);
# lane slot % 4 of the output block becomes (x >> 8) * 2^-24.
_PHILOX_M0 = np.uint64(0xD2511F53)
_PHILOX_M1 = np.uint64(0xCD9E8D57)
_PHILOX_W0 = np.uint32(0x9E3779B9)
_PHILOX_W1 = np.uint32(0xBB67AE85)
PHILOX_TAG = 0x53504543


def philox4x32_10(ctr: np.ndarray, key: Tuple[int, int]) -> np.ndarray:
    """ctr: uint32 [..., 4] -> uint32 [..., 4]."""
    c = [ctr[..., i].astype(np.uint64) for i in range(4)]
    k0 = np.uint32(key[0] & 0xFFFFFFFF)
    k1 = np.uint32(key[1] & 0xFFFFFFFF)
    mask = np.uint64(0xFFFFFFFF)
    for _ in range(10):
        p0 = _PHILOX_M0 * c[0]
        p1 = _PHILOX_M1 * c[2]
        hi0, lo0 = p0 >> np.uint64(32), p0 & mask
        hi1, lo1 = p1 >> np.uint64(32), p1 & mask
        c = [hi1 ^ c[1] ^ np.uint64(k0), lo1, hi0 ^ c[3] ^ np.uint64(k1), lo0]
        k0 = np.uint32((int(k0) + int(_PHILOX_W0)) & 0xFFFFFFFF)
        k1 = np.uint32((int(k1) + int(_PHILOX_W1)) & 0xFFFFFFFF)
    return np.stack([x.astype(np.uint32) for x in c], axis=-1)


def philox_uniforms(seed: int, B: int, n_rounds: int, slots: int) -> np.ndarray:
    """float32 [B, n_rounds, slots] in [0, 1)."""
    nblk = (slots + 3) // 4
    b, r, s = np.meshgrid(np.arange(B, dtype=np.uint32), np.arange(n_rounds, dtype=np.uint32),
                          np.arange(nblk, dtype=np.uint32), indexing="ij")
    ctr = np.stack([s, r, b, np.full_like(b, PHILOX_TAG)], axis=-1)
    x = philox4x32_10(ctr, (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF))
    x = x.reshape(B, n_rounds, nblk * 4)[:, :, :slots]
    return ((x >> np.uint32(8)).astype(np.float32) * np.float32(2.0 ** -24)).astype(np.float32)


# ---------------------------------------------------------------------------
# The five BASELINE configurations (shapes only; dtype/batch/sampling settings
# live with the benchmark and the tests).
@dataclass(frozen=True)
class Workload:
    name: str
    target: ModelShape
    draft_layers: int
    batch: int
    prompt_len: int
    max_new: int
    lookahead: int
    temperature: float
    weights_int8: bool
    act_bf16: bool
    kv_mode: int = 0  # 0 fp32, 1 bf16, 2 int8
    tree: tuple = ()  # token-tree branching per level (tree speculation), () for a chain


def _shape(V, d, H, F, L, max_seq, arch=ARCH_REF):
    return ModelShape(vocab=V, d_model=d, n_heads=H, d_ff=F, n_layers=L, max_seq_len=max_seq, arch=arch)


def workload(name: str, arch: int = ARCH_REF) -> Workload:
    # max_seq_len leaves room for the reference's draft catch-up drift (the draft
    # cache grows by one extra position per rejected round).
    if name == "tiny":
        return Workload("tiny", _shape(2048, 256, 4, 1024, 4, 32 + 2 * 128 + 8, arch), 1, 1, 32, 128, 4, 0.0, False, False)
    if name == "int8":
        return Workload("int8", _shape(2048, 256, 4, 1024, 4, 64 + 2 * 256 + 8, arch), 1, 8, 64, 256, 4, 1.0, True, False)
    if name == "medium":
        return Workload("medium", _shape(32000, 768, 12, 3072, 12, 256 + 2 * 256 + 16, arch), 2, 32, 256, 256, 6, 0.8, True, True, 1)
    if name == "tree":
        # config-3 models, 64 requests, 512-token prompts,
        # a 4/3/2/1 tree (64 nodes); 256 new tokens
        return Workload("tree", _shape(32000, 768, 12, 3072, 12, 512 + 256 + 80, arch), 2, 64, 512, 256, 4, 1.0, True, True,
                        1, (4, 3, 2, 1))
    if name == "large":
        return Workload("large", _shape(32000, 4096, 32, 11008, 32, 2048 + 2 * 512 + 8, arch), 4, 256, 2048, 512, 4, 1.0, True, True, 1)
    raise KeyError(name)
