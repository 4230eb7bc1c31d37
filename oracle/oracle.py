"""TEST INFRASTRUCTURE ONLY: ctypes access to the two CPU checkers.

* ``Reference`` drives the unmodified reference library built by
  oracle/Makefile into oracle/_ref/libnnref.so (see oracle/ref_shim.cpp).
* ``Oracle`` drives the CPU restatement oracle/specdec_oracle.cpp
  (oracle/_build/liboracle.so), which adds batching, host-supplied uniforms,
  int8 weights, bf16 rounding and the draft catch-up switch.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs import this module.  The product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from typing import List, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_SO = os.path.join(HERE, "_ref", "libnnref.so")
# the reference library with the B200 dispatch of oracle/binding/ (make bind)
REF_CUDA_SO = os.path.join(HERE, "_ref", "libnnref_cuda.so")
ORACLE_SO = os.path.join(HERE, "_build", "liboracle.so")


def reference_tree() -> str:
    """The reference source tree used to compile oracle/_ref: $NN_REFERENCE_SRC,
    else a `reference` checkout beside this repository ("" when neither exists)."""
    env = os.environ.get("NN_REFERENCE_SRC", "")
    if env:
        return env if os.path.isdir(env) else ""
    sib = os.path.normpath(os.path.join(HERE, "..", "..", "reference"))
    return sib if os.path.isdir(os.path.join(sib, "src", "nn")) else ""

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")


def build(ref: bool = True) -> None:
    """Compile the restatement (and the reference shim when its sources exist)."""
    targets = ["oracle"]
    tree = reference_tree() if ref else ""
    if tree:
        targets += ["ref", f"REF={tree}"]
        # the reference with the B200 dispatch, once the product library is built
        if os.path.exists(os.path.join(HERE, "..", "neural-network_b200", "specdec_b200", "libspecdec_b200.so")):
            targets.insert(-1, "bind")
    subprocess.run(["make", "-s", "-C", HERE] + targets, check=True)


def reference_available() -> bool:
    return os.path.exists(REF_SO)


# ---------------------------------------------------------------------------
class _RefLib:
    _libs = {}

    @classmethod
    def get(cls, cuda: bool = False):
        if cuda not in cls._libs:
            lib = C.CDLL(REF_CUDA_SO if cuda else REF_SO)
            lib.nnref_last_error.restype = C.c_char_p
            lib.nnref_decoder_new.restype = C.c_void_p
            lib.nnref_decoder_new.argtypes = [C.c_size_t] * 6
            lib.nnref_decoder_free.argtypes = [C.c_void_p]
            lib.nnref_num_params.argtypes = [C.c_void_p]
            lib.nnref_param_numel.restype = C.c_size_t
            lib.nnref_param_numel.argtypes = [C.c_void_p, C.c_int]
            lib.nnref_set_param.argtypes = [C.c_void_p, C.c_int, _f32p, C.c_size_t]
            lib.nnref_get_param.argtypes = [C.c_void_p, C.c_int, _f32p, C.c_size_t]
            lib.nnref_set_requires_grad.argtypes = [C.c_void_p, C.c_int]
            lib.nnref_forward.argtypes = [C.c_void_p, _i64p, C.c_size_t, _f32p]
            lib.nnref_save_weights.argtypes = [C.c_void_p, C.c_char_p]
            lib.nnref_load_weights.argtypes = [C.c_void_p, C.c_char_p]
            lib.nnref_generate.argtypes = [C.c_void_p, _i64p, C.c_size_t, C.c_size_t, _i64p, C.c_size_t,
                                           C.POINTER(C.c_size_t)]
            lib.nnref_generate_advanced.argtypes = [C.c_void_p, _i64p, C.c_size_t, C.c_size_t, C.c_float,
                                                    C.c_size_t, C.c_float, C.c_uint, C.c_int, _i64p,
                                                    C.c_size_t, C.POINTER(C.c_size_t)]
            lib.nnref_generate_speculative.argtypes = [C.c_void_p, C.c_void_p, _i64p, C.c_size_t, C.c_size_t,
                                                       C.c_size_t, C.c_float, C.c_size_t, C.c_float, C.c_uint,
                                                       C.c_int, _i64p, C.c_size_t, C.POINTER(C.c_size_t)]
            lib.nnref_rope.argtypes = [_f32p] + [C.c_size_t] * 5 + [_f32p]
            lib.nnref_quantize_int8.argtypes = [_f32p, C.c_size_t, C.c_size_t, _f32p, _i8p, _f32p]
            if cuda:
                lib.nnref_cuda_backend_new.restype = C.c_void_p
                lib.nnref_cuda_backend_new.argtypes = [C.c_void_p, C.c_int]
                lib.nnref_cuda_backend_free.argtypes = [C.c_void_p]
                lib.nnref_cuda_backend_launches.restype = C.c_longlong
                lib.nnref_cuda_backend_launches.argtypes = [C.c_void_p]
                lib.nnref_decoder_new_on.restype = C.c_void_p
                lib.nnref_decoder_new_on.argtypes = [C.c_void_p] + [C.c_size_t] * 6
            cls._libs[cuda] = lib
        return cls._libs[cuda]


def _ref_check(rc: int, lib=None) -> None:
    if rc != 0:
        raise RuntimeError((lib or _RefLib.get()).nnref_last_error().decode())


def bound_reference_available() -> bool:
    return os.path.exists(REF_CUDA_SO)


class _SpecModelCfg(C.Structure):  # specdec_model_config (include/specdec.h)
    _fields_ = [(n, C.c_int32) for n in ("vocab_size", "d_model", "n_heads", "n_kv_heads", "d_ff", "n_layers",
                                         "max_seq_len", "arch")]


class _SpecCfg(C.Structure):  # specdec_config (include/specdec.h)
    _fields_ = [("target", _SpecModelCfg), ("draft", _SpecModelCfg)] + [
        (n, C.c_int32) for n in ("draft_shares_target", "weight_dtype", "act_dtype", "kv_dtype", "max_batch",
                                 "max_lookahead", "max_prompt_len", "max_tree_nodes", "kv_pages")]


class CudaSpecBackendRef:
    """A CudaSpecBackend (oracle/binding/cuda_spec_backend.hpp) in the
    reference library built with the B200 dispatch: decoders constructed on it
    (Reference(..., backend=this)) run generate_speculative and
    generate_advanced through libspecdec_b200.so.  fp32 weights, activations
    and cache (a quantized_cache call switches the cache to int8)."""

    def __init__(self, target_shape, draft_shape, device: int = 0, max_prompt_len: int = 0):
        self.lib = _RefLib.get(cuda=True)

        def mc(m):
            return _SpecModelCfg(m.vocab, m.d_model, m.n_heads, m.kv_heads, m.d_ff, m.n_layers, m.max_seq_len, 0)

        cfg = _SpecCfg(mc(target_shape), mc(draft_shape), 0, 0, 0, 0, 1, 8,
                       max_prompt_len or target_shape.max_seq_len, 0)
        self.h = self.lib.nnref_cuda_backend_new(C.byref(cfg), device)
        if not self.h:
            _ref_check(-1, self.lib)

    def launches(self) -> int:
        return int(self.lib.nnref_cuda_backend_launches(self.h))

    def close(self):
        if getattr(self, "h", None):
            self.lib.nnref_cuda_backend_free(self.h)
            self.h = None


class Reference:
    """One reference ``TransformerDecoder`` with injected weights."""

    def __init__(self, shape, params: Sequence[np.ndarray], requires_grad: bool = True,
                 backend: Optional[CudaSpecBackendRef] = None):
        if shape.arch != 0 or shape.kv_heads != shape.n_heads:
            raise ValueError("the reference TransformerDecoder is the post-LN SwiGLU MHA model")
        lib = backend.lib if backend is not None else _RefLib.get()
        self._lib = lib
        self.backend = backend  # kept alive as long as the decoder
        self.shape = shape
        dims = (shape.vocab, shape.d_model, shape.n_heads, shape.d_ff, shape.n_layers, shape.max_seq_len)
        self.h = lib.nnref_decoder_new_on(backend.h, *dims) if backend is not None else lib.nnref_decoder_new(*dims)
        if not self.h:
            _ref_check(-1, lib)
        n = lib.nnref_num_params(self.h)
        if n != len(params):
            raise ValueError(f"reference has {n} parameters, got {len(params)}")
        for i, p in enumerate(params):
            a = np.ascontiguousarray(p, np.float32).ravel()
            _ref_check(lib.nnref_set_param(self.h, i, a, a.size), lib)
        lib.nnref_set_requires_grad(self.h, 1 if requires_grad else 0)

    def _chk(self, rc: int) -> None:
        _ref_check(rc, self._lib)

    def __del__(self):
        if getattr(self, "h", None):
            self._lib.nnref_decoder_free(self.h)
            self.h = None

    def forward(self, tokens: Sequence[int]) -> np.ndarray:
        t = np.ascontiguousarray(tokens, np.int64)
        out = np.zeros((t.size, self.shape.vocab), np.float32)
        self._chk(self._lib.nnref_forward(self.h, t, t.size, out))
        return out

    def save_weights(self, path: str) -> None:
        """Layer::save_weights: the reference's NETW v1 parameter file."""
        self._chk(self._lib.nnref_save_weights(self.h, os.fsencode(path)))

    def load_weights(self, path: str) -> None:
        self._chk(self._lib.nnref_load_weights(self.h, os.fsencode(path)))

    def _tokens_call(self, fn, prompt, max_new, *args):
        p = np.ascontiguousarray(prompt, np.int64)
        out = np.zeros(p.size + max_new, np.int64)
        n = C.c_size_t(0)
        self._chk(fn(self.h, *args[:1], p, p.size, max_new, *args[1:], out, out.size, C.byref(n)))
        return out[: n.value]

    def generate(self, prompt, max_new):
        lib = self._lib
        p = np.ascontiguousarray(prompt, np.int64)
        out = np.zeros(p.size + max_new, np.int64)
        n = C.c_size_t(0)
        self._chk(lib.nnref_generate(self.h, p, p.size, max_new, out, out.size, C.byref(n)))
        return out[: n.value]

    def generate_advanced(self, prompt, max_new, temperature=1.0, top_k=0, top_p=1.0, seed=42,
                          use_kv_cache=True):
        lib = self._lib
        p = np.ascontiguousarray(prompt, np.int64)
        out = np.zeros(p.size + max_new, np.int64)
        n = C.c_size_t(0)
        self._chk(lib.nnref_generate_advanced(self.h, p, p.size, max_new, temperature, top_k, top_p,
                                               seed, 1 if use_kv_cache else 0, out, out.size, C.byref(n)))
        return out[: n.value]

    def generate_speculative(self, draft: "Reference", prompt, max_new, lookahead=4, temperature=1.0,
                             top_k=0, top_p=1.0, seed=42, quantized_cache=False):
        lib = self._lib
        p = np.ascontiguousarray(prompt, np.int64)
        out = np.zeros(p.size + max_new, np.int64)
        n = C.c_size_t(0)
        self._chk(lib.nnref_generate_speculative(self.h, draft.h, p, p.size, max_new, lookahead,
                                                  temperature, top_k, top_p, seed,
                                                  1 if quantized_cache else 0, out, out.size, C.byref(n)))
        return out[: n.value]


def ref_rope(x: np.ndarray, s_past: int) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    B, H, S, D = x.shape
    out = np.zeros_like(x)
    _ref_check(_RefLib.get().nnref_rope(x, B, H, S, D, s_past, out))
    return out


def ref_quantize_int8(w: np.ndarray):
    w = np.ascontiguousarray(w, np.float32)
    i, o = w.shape
    s = np.zeros(o, np.float32)
    q = np.zeros((i, o), np.int8)
    dq = np.zeros((i, o), np.float32)
    _ref_check(_RefLib.get().nnref_quantize_int8(w, i, o, s, q, dq))
    return s, q, dq


# ---------------------------------------------------------------------------
class _ModelCfg(C.Structure):
    _fields_ = [("vocab", C.c_int32), ("d_model", C.c_int32), ("n_heads", C.c_int32),
                ("n_kv_heads", C.c_int32), ("d_ff", C.c_int32), ("n_layers", C.c_int32),
                ("max_seq_len", C.c_int32), ("arch", C.c_int32)]


class _Numerics(C.Structure):
    _fields_ = [("act_bf16", C.c_int32), ("kv_mode", C.c_int32)]


class _SpecParams(C.Structure):
    _fields_ = [("max_new", C.c_int32), ("lookahead", C.c_int32), ("temperature", C.c_float),
                ("top_k", C.c_int32), ("top_p", C.c_float), ("rng_mode", C.c_int32),
                ("seed", C.c_uint32), ("uniforms", C.c_void_p), ("n_rounds", C.c_int32),
                ("catchup", C.c_int32), ("num", _Numerics), ("cache_cap", C.c_int32)]


class _TreeParams(C.Structure):
    _fields_ = [("depth", C.c_int32), ("branch", C.c_int32 * 8)]


def tree_slots(branching) -> int:
    """Uniform slots per round of tree speculation: depth * max branch + 1."""
    return len(branching) * max(branching) + 1


def tree_nodes(branching) -> int:
    n, level = 0, 1
    for b in branching:
        level *= b
        n += level
    return n


class _OracleLib:
    _lib = None

    @classmethod
    def get(cls):
        if cls._lib is None:
            lib = C.CDLL(ORACLE_SO)
            lib.oc_last_error.restype = C.c_char_p
            lib.oc_model_new.restype = C.c_void_p
            lib.oc_model_new.argtypes = [C.POINTER(_ModelCfg)]
            lib.oc_model_free.argtypes = [C.c_void_p]
            lib.oc_model_num_params.argtypes = [C.c_void_p]
            lib.oc_model_param_numel.restype = C.c_int64
            lib.oc_model_param_numel.argtypes = [C.c_void_p, C.c_int]
            lib.oc_model_set_param.argtypes = [C.c_void_p, C.c_int, _f32p, C.c_int64]
            lib.oc_model_get_param.argtypes = [C.c_void_p, C.c_int, _f32p, C.c_int64]
            lib.oc_model_quantize_int8.argtypes = [C.c_void_p]
            lib.oc_forward.argtypes = [C.c_void_p, C.POINTER(_Numerics), _i64p, C.c_int, _f32p]
            lib.oc_forward_chunked.argtypes = [C.c_void_p, C.POINTER(_Numerics), _i64p, _i32p, C.c_int, _f32p]
            lib.oc_generate_speculative.argtypes = [C.c_void_p, C.c_void_p, C.POINTER(_SpecParams), _i64p,
                                                    C.c_int, C.c_int, _i64p, _i64p, C.c_void_p, C.c_int]
            lib.oc_generate_tree.argtypes = [C.c_void_p, C.c_void_p, C.POINTER(_SpecParams), C.POINTER(_TreeParams),
                                             _i64p, C.c_int, C.c_int, _i64p, _i64p, C.c_void_p, C.c_int]
            lib.oc_generate_advanced.argtypes = [C.c_void_p, C.POINTER(_Numerics), _i64p, C.c_int, C.c_int,
                                                 C.c_float, C.c_int, C.c_float, C.c_uint32, _i64p]
            lib.oc_generate_ar.argtypes = [C.c_void_p, C.POINTER(_Numerics), _i64p, C.c_int, C.c_int, C.c_int,
                                           C.c_float, C.c_int, C.c_float, C.c_int, C.c_uint32, C.c_void_p, C.c_int,
                                           _i64p, C.c_void_p]
            lib.oc_get_probs.argtypes = [_f32p, C.c_int, C.c_float, C.c_int, C.c_float, _f32p]
            lib.oc_rope.argtypes = [_f32p, C.c_int, C.c_int, _i32p, _f32p]
            lib.oc_mt19937.argtypes = [C.c_uint32, C.c_int, _u32p]
            cls._lib = lib
        return cls._lib


def _oc_check(rc: int) -> None:
    if rc != 0:
        raise RuntimeError(_OracleLib.get().oc_last_error().decode())


class Oracle:
    """One model in the CPU restatement."""

    def __init__(self, shape, params: Sequence[np.ndarray], int8: bool = False):
        lib = _OracleLib.get()
        self.shape = shape
        cfg = _ModelCfg(shape.vocab, shape.d_model, shape.n_heads, shape.kv_heads, shape.d_ff,
                        shape.n_layers, shape.max_seq_len, shape.arch)
        self.h = lib.oc_model_new(C.byref(cfg))
        if not self.h:
            _oc_check(-1)
        n = lib.oc_model_num_params(self.h)
        if n != len(params):
            raise ValueError(f"oracle model has {n} parameters, got {len(params)}")
        for i, p in enumerate(params):
            a = np.ascontiguousarray(p, np.float32).ravel()
            _oc_check(lib.oc_model_set_param(self.h, i, a, a.size))
        if int8:
            _oc_check(lib.oc_model_quantize_int8(self.h))

    def __del__(self):
        if getattr(self, "h", None):
            _OracleLib.get().oc_model_free(self.h)
            self.h = None

    def param(self, i: int) -> np.ndarray:
        lib = _OracleLib.get()
        n = lib.oc_model_param_numel(self.h, i)
        out = np.zeros(n, np.float32)
        _oc_check(lib.oc_model_get_param(self.h, i, out, n))
        return out

    def forward(self, tokens, act_bf16=False, kv_mode=0) -> np.ndarray:
        t = np.ascontiguousarray(tokens, np.int64)
        out = np.zeros((t.size, self.shape.vocab), np.float32)
        nm = _Numerics(1 if act_bf16 else 0, kv_mode)
        _oc_check(_OracleLib.get().oc_forward(self.h, C.byref(nm), t, t.size, out))
        return out

    def forward_chunked(self, tokens, chunks, act_bf16=False, kv_mode=0) -> np.ndarray:
        t = np.ascontiguousarray(tokens, np.int64)
        ch = np.ascontiguousarray(chunks, np.int32)
        assert int(ch.sum()) == t.size
        out = np.zeros((t.size, self.shape.vocab), np.float32)
        nm = _Numerics(1 if act_bf16 else 0, kv_mode)
        _oc_check(_OracleLib.get().oc_forward_chunked(self.h, C.byref(nm), t, ch, ch.size, out))
        return out

    def generate_advanced(self, prompt, max_new, temperature=1.0, top_k=0, top_p=1.0, seed=42,
                          act_bf16=False, kv_mode=0):
        p = np.ascontiguousarray(prompt, np.int64)
        out = np.zeros(p.size + max_new, np.int64)
        nm = _Numerics(1 if act_bf16 else 0, kv_mode)
        _oc_check(_OracleLib.get().oc_generate_advanced(self.h, C.byref(nm), p, p.size, max_new,
                                                        temperature, top_k, top_p, seed, out))
        return out


def oracle_generate_ar(model: Oracle, prompts: np.ndarray, max_new: int, temperature: float = 1.0, top_k: int = 0,
                       top_p: float = 1.0, seed: int = 42, uniforms: Optional[np.ndarray] = None,
                       act_bf16: bool = False, kv_mode: int = 0):
    """generate_advanced with the KV cache (src/nn/layer.cpp:1239-1380) for B
    requests: request b uses mt19937(seed + b), or uniforms[b][step][0].
    Returns (tokens [B, S + max_new], margins [B, max_new] per token)."""
    p = np.ascontiguousarray(np.atleast_2d(prompts), np.int64)
    B, S = p.shape
    out = np.zeros((B, S + max_new), np.int64)
    margins = np.zeros((B, max(1, max_new)), np.float64)
    nm = _Numerics(1 if act_bf16 else 0, kv_mode)
    u = None if uniforms is None else np.ascontiguousarray(uniforms, np.float32)
    _oc_check(_OracleLib.get().oc_generate_ar(model.h, C.byref(nm), p, B, S, max_new, temperature, top_k, top_p,
                                              0 if u is None else 1, seed & 0xFFFFFFFF,
                                              None if u is None else u.ctypes.data,
                                              0 if u is None else u.shape[1], out, margins.ctypes.data))
    return out, margins


def oracle_generate_speculative(target: Oracle, draft: Oracle, prompts: np.ndarray, max_new: int,
                                lookahead: int = 4, temperature: float = 1.0, top_k: int = 0,
                                top_p: float = 1.0, seed: int = 42,
                                uniforms: Optional[np.ndarray] = None, catchup: int = 0,
                                act_bf16: bool = False, kv_mode: int = 0, cache_cap: int = 0,
                                n_threads: int = 0):
    """Returns (tokens [B, S+max_new], stats [B, 4], margins [B, max_new])."""
    prompts = np.ascontiguousarray(np.atleast_2d(prompts), np.int64)
    B, S = prompts.shape
    out = np.zeros((B, S + max_new), np.int64)
    stats = np.zeros((B, 4), np.int64)
    margins = np.full((B, max_new), np.inf, np.float64)
    keep = None
    if uniforms is not None:
        keep = np.ascontiguousarray(uniforms, np.float32)
        assert keep.shape[0] == B and keep.shape[2] == 2 * lookahead + 1
        uptr, n_rounds, mode = keep.ctypes.data, keep.shape[1], 1
    else:
        uptr, n_rounds, mode = None, 0, 0
    sp = _SpecParams(max_new, lookahead, temperature, top_k, top_p, mode, seed & 0xFFFFFFFF, uptr,
                     n_rounds, catchup, _Numerics(1 if act_bf16 else 0, kv_mode), cache_cap)
    _oc_check(_OracleLib.get().oc_generate_speculative(target.h, draft.h, C.byref(sp), prompts, B, S,
                                                       out, stats, margins.ctypes.data, n_threads))
    del keep
    return out, stats, margins


def oracle_generate_tree(target: Oracle, draft: Oracle, prompts: np.ndarray, max_new: int, branching,
                         temperature: float = 1.0, top_k: int = 0, top_p: float = 1.0, seed: int = 42,
                         uniforms: Optional[np.ndarray] = None, act_bf16: bool = False, kv_mode: int = 0,
                         cache_cap: int = 0, n_threads: int = 0):
    """Tree speculation (oracle/specdec_oracle.cpp: tree_one).  Returns
    (tokens [B, S+max_new], stats [B, 4] = rounds, tree nodes drafted, accepted, rejections,
    margins [B, max_new])."""
    prompts = np.ascontiguousarray(np.atleast_2d(prompts), np.int64)
    B, S = prompts.shape
    out = np.zeros((B, S + max_new), np.int64)
    stats = np.zeros((B, 4), np.int64)
    margins = np.full((B, max_new), np.inf, np.float64)
    keep = None
    if uniforms is not None:
        keep = np.ascontiguousarray(uniforms, np.float32)
        assert keep.shape[0] == B and keep.shape[2] == tree_slots(branching)
        uptr, n_rounds, mode = keep.ctypes.data, keep.shape[1], 1
    else:
        uptr, n_rounds, mode = None, 0, 0
    sp = _SpecParams(max_new, len(branching), temperature, top_k, top_p, mode, seed & 0xFFFFFFFF, uptr,
                     n_rounds, 1, _Numerics(1 if act_bf16 else 0, kv_mode), cache_cap)
    tp = _TreeParams(len(branching), (C.c_int32 * 8)(*list(branching)))
    _oc_check(_OracleLib.get().oc_generate_tree(target.h, draft.h, C.byref(sp), C.byref(tp), prompts, B, S,
                                                out, stats, margins.ctypes.data, n_threads))
    del keep
    return out, stats, margins


def oracle_get_probs(logits: np.ndarray, temperature: float, top_k: int = 0, top_p: float = 1.0):
    l = np.ascontiguousarray(logits, np.float32)
    out = np.zeros_like(l)
    _oc_check(_OracleLib.get().oc_get_probs(l, l.size, temperature, top_k, top_p, out))
    return out


def oracle_rope(rows: np.ndarray, pos: np.ndarray) -> np.ndarray:
    r = np.ascontiguousarray(rows, np.float32)
    p = np.ascontiguousarray(pos, np.int32)
    out = np.zeros_like(r)
    _oc_check(_OracleLib.get().oc_rope(r, r.shape[0], r.shape[1], p, out))
    return out


def mt19937(seed: int, n: int) -> np.ndarray:
    out = np.zeros(n, np.uint32)
    _OracleLib.get().oc_mt19937(seed & 0xFFFFFFFF, n, out)
    return out
