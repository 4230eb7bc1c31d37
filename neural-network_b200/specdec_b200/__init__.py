"""Python binding of the B200 speculative-decoding backend (libspecdec_b200.so).

Mirrors the reference's entry point
``TransformerDecoder::generate_speculative(draft, prompt, max_new_tokens,
lookahead, temperature, top_k, top_p, seed, quantized_cache)``
(include/nn/layer.hpp:318-323, src/nn/layer.cpp:1382-1661) over the C ABI of
include/specdec.h, batched over B requests.  Failures raise ``SpecDecError``
(a RuntimeError, as the reference throws std::runtime_error).

There is no CPU fallback: if the shared library is missing or cannot be
loaded, importing the engine raises.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional, Sequence, Tuple

import numpy as np

from .synth import ARCH_CFG, ARCH_REF, ModelShape  # noqa: F401

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libspecdec_b200.so")

F32, BF16, INT8 = 0, 1, 2
TARGET, DRAFT = 0, 1
RNG_MT19937, RNG_HOST_UNIFORM = 0, 1
CATCHUP_REF, CATCHUP_CORRECT = 0, 1

STATUS = {0: "OK", 1: "ERR_INVALID", 2: "ERR_CUDA", 3: "ERR_OOM", 4: "ERR_SEQ_LEN", 5: "ERR_UNSUPPORTED",
          6: "ERR_STATE", 7: "ERR_RNG"}

# Every symbol include/specdec.h declares.
EXPORTS = ("specdec_create", "specdec_destroy", "specdec_last_error", "specdec_load_params",
           "specdec_generate", "specdec_generate_device", "specdec_stream", "specdec_forward_logits",
           "specdec_philox_uniforms", "specdec_last_launch_count", "specdec_forward_logits_noalloc",
           "specdec_time_linear", "specdec_generate_tree", "specdec_generate_tree_device", "specdec_tp_unique_id",
           "specdec_create_tp", "specdec_generate_ar", "specdec_generate_ar_device", "specdec_load_netw",
           "specdec_prefill", "specdec_prefill_device", "specdec_step", "specdec_step_device",
           "specdec_session_tokens", "specdec_time_attention", "specdec_load_params_device")

# linear layers of specdec_time_linear
LIN_QKV, LIN_OPROJ, LIN_FFN_IN, LIN_FFN_OUT, LIN_HEAD = 0, 1, 2, 3, 4


class SpecDecError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS.get(code, code)}: {msg}")
        self.code = code


class _ModelConfig(C.Structure):
    _fields_ = [("vocab_size", C.c_int32), ("d_model", C.c_int32), ("n_heads", C.c_int32),
                ("n_kv_heads", C.c_int32), ("d_ff", C.c_int32), ("n_layers", C.c_int32),
                ("max_seq_len", C.c_int32), ("arch", C.c_int32)]


class _Config(C.Structure):
    _fields_ = [("target", _ModelConfig), ("draft", _ModelConfig), ("draft_shares_target", C.c_int32),
                ("weight_dtype", C.c_int32), ("act_dtype", C.c_int32), ("kv_dtype", C.c_int32),
                ("max_batch", C.c_int32), ("max_lookahead", C.c_int32), ("max_prompt_len", C.c_int32),
                ("max_tree_nodes", C.c_int32), ("kv_pages", C.c_int32)]


class _Tree(C.Structure):
    _fields_ = [("depth", C.c_int32), ("branch", C.c_int32 * 8)]


class _GenParams(C.Structure):
    _fields_ = [("max_new_tokens", C.c_int32), ("lookahead", C.c_int32), ("temperature", C.c_float),
                ("top_k", C.c_int32), ("top_p", C.c_float), ("rng_mode", C.c_int32), ("seed", C.c_uint32),
                ("uniforms", C.c_void_p), ("uniform_rounds", C.c_int32), ("draft_catchup", C.c_int32)]


_lib = None


def load_library(path: str = LIB_PATH):
    """Loads the shared library (raises if it is absent: no fallback path)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing; build it with neural-network_b200/build.py")
    lib = C.CDLL(path)
    lib.specdec_create.argtypes = [C.POINTER(_Config), C.c_int, C.POINTER(C.c_void_p)]
    lib.specdec_destroy.argtypes = [C.c_void_p]
    lib.specdec_last_error.restype = C.c_char_p
    lib.specdec_last_error.argtypes = [C.c_void_p]
    lib.specdec_load_params.argtypes = [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_void_p),
                                        C.POINTER(C.c_int64)]
    lib.specdec_generate.argtypes = [C.c_void_p, C.POINTER(_GenParams), C.c_void_p, C.c_int, C.c_int,
                                     C.c_void_p, C.c_void_p]
    lib.specdec_generate_device.argtypes = [C.c_void_p, C.POINTER(_GenParams), C.c_void_p, C.c_int, C.c_int,
                                            C.c_void_p, C.c_void_p]
    lib.specdec_load_netw.argtypes = [C.c_void_p, C.c_int, C.c_char_p]
    lib.specdec_load_params_device.argtypes = lib.specdec_load_params.argtypes
    lib.specdec_prefill.argtypes = [C.c_void_p, C.POINTER(_GenParams), C.c_void_p, C.c_int, C.c_int]
    lib.specdec_prefill_device.argtypes = lib.specdec_prefill.argtypes
    lib.specdec_step.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
    lib.specdec_step_device.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]
    lib.specdec_session_tokens.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p]
    lib.specdec_generate_ar.argtypes = lib.specdec_generate.argtypes
    lib.specdec_generate_ar_device.argtypes = lib.specdec_generate_device.argtypes
    lib.specdec_stream.restype = C.c_void_p
    lib.specdec_stream.argtypes = [C.c_void_p]
    lib.specdec_forward_logits.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p]
    lib.specdec_philox_uniforms.argtypes = [C.c_uint64, C.c_int, C.c_int, C.c_int, C.c_void_p]
    lib.specdec_forward_logits_noalloc.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                                   C.c_void_p, C.c_void_p]
    lib.specdec_last_launch_count.restype = C.c_int64
    lib.specdec_last_launch_count.argtypes = [C.c_void_p]
    lib.specdec_generate_tree.argtypes = [C.c_void_p, C.POINTER(_GenParams), C.POINTER(_Tree), C.c_void_p, C.c_int,
                                          C.c_int, C.c_void_p, C.c_void_p]
    lib.specdec_generate_tree_device.argtypes = [C.c_void_p, C.POINTER(_GenParams), C.POINTER(_Tree), C.c_void_p,
                                                 C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    lib.specdec_tp_unique_id.argtypes = [C.c_void_p]
    lib.specdec_create_tp.argtypes = [C.POINTER(_Config), C.c_int, C.c_int, C.c_int, C.c_void_p,
                                      C.POINTER(C.c_void_p)]
    lib.specdec_time_linear.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                        C.c_size_t, C.POINTER(C.c_float), C.POINTER(C.c_double)]
    lib.specdec_time_attention.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_size_t,
                                           C.POINTER(C.c_float), C.POINTER(C.c_double)]
    _lib = lib
    return lib


def _mcfg(m: ModelShape) -> _ModelConfig:
    return _ModelConfig(m.vocab, m.d_model, m.n_heads, m.n_kv_heads, m.d_ff, m.n_layers, m.max_seq_len, m.arch)


def philox_uniforms(seed: int, B: int, rounds: int, slots: int) -> np.ndarray:
    lib = load_library()
    out = np.zeros((B, rounds, slots), np.float32)
    rc = lib.specdec_philox_uniforms(seed, B, rounds, slots, out.ctypes.data)
    if rc:
        raise SpecDecError(rc, "philox")
    return out


def tp_unique_id() -> bytes:
    """The 128-byte NCCL id that all ranks of a tensor-parallel group pass to
    Engine(tp_rank=..., tp_world=..., tp_id=...)."""
    lib = load_library()
    buf = C.create_string_buffer(128)
    rc = lib.specdec_tp_unique_id(buf)
    if rc:
        raise SpecDecError(rc, lib.specdec_last_error(None).decode())
    return buf.raw


class Engine:
    """A target/draft pair on one B200 (one handle of the C ABI)."""

    def __init__(self, target: ModelShape, draft_layers: Optional[int] = None, draft: Optional[ModelShape] = None,
                 weight_dtype: int = F32, act_dtype: int = F32, kv_dtype: int = F32, max_batch: int = 1,
                 max_lookahead: int = 4, max_prompt_len: int = 128, device: int = 0, max_tree_nodes: int = 0,
                 tp_rank: int = 0, tp_world: int = 1, tp_id: Optional[bytes] = None, kv_pages: int = 0):
        lib = load_library()
        shares = draft is None
        if shares and draft_layers is None:
            raise ValueError("give draft_layers (shared draft) or a draft shape")
        dshape = target.with_layers(draft_layers) if shares else draft
        cfg = _Config(_mcfg(target), _mcfg(dshape), 1 if shares else 0, weight_dtype, act_dtype, kv_dtype,
                      max_batch, max_lookahead, max_prompt_len, max_tree_nodes, kv_pages)
        h = C.c_void_p()
        if tp_world > 1:
            uid = C.create_string_buffer(bytes(tp_id), 128)
            rc = lib.specdec_create_tp(C.byref(cfg), device, tp_rank, tp_world, uid, C.byref(h))
        else:
            rc = lib.specdec_create(C.byref(cfg), device, C.byref(h))
        if rc:
            raise SpecDecError(rc, lib.specdec_last_error(None).decode())
        self._lib = lib
        self.h = h
        self.target = target
        self.draft = dshape
        self.shares = shares
        self.max_batch = max_batch
        self.max_lookahead = max_lookahead

    def close(self):
        if getattr(self, "h", None):
            self._lib.specdec_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def _check(self, rc: int):
        if rc:
            raise SpecDecError(rc, self._lib.specdec_last_error(self.h).decode())

    def load_params(self, role: int, params: Sequence[np.ndarray]) -> None:
        arrs = [np.ascontiguousarray(p, np.float32) for p in params]
        ptrs = (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])
        nums = (C.c_int64 * len(arrs))(*[a.size for a in arrs])
        self._check(self._lib.specdec_load_params(self.h, role, len(arrs), ptrs, nums))

    def load_params_device(self, role: int, tensors) -> None:
        """load_params from fp32 device tensors (e.g. torch CUDA tensors, any
        object with data_ptr() and numel()) on this engine's device: quantised
        and transposed on the device, no host copy."""
        ptrs = (C.c_void_p * len(tensors))(*[t.data_ptr() for t in tensors])
        nums = (C.c_int64 * len(tensors))(*[t.numel() for t in tensors])
        self._check(self._lib.specdec_load_params_device(self.h, role, len(tensors), ptrs, nums))

    def load_weights(self, role: int, path: str) -> None:
        """Layer::load_weights: the model's parameters from a NETW v1 file (the
        reference's serialization format, src/core/serialization.cpp:49-107)."""
        self._check(self._lib.specdec_load_netw(self.h, role, os.fsencode(path)))

    def _params(self, max_new, lookahead, temperature, top_k, top_p, seed, uniforms, draft_catchup):
        if uniforms is not None:
            u = np.ascontiguousarray(uniforms, np.float32)
            return _GenParams(max_new, lookahead, temperature, top_k, top_p, RNG_HOST_UNIFORM, seed & 0xFFFFFFFF,
                              u.ctypes.data, u.shape[1], draft_catchup), u
        return _GenParams(max_new, lookahead, temperature, top_k, top_p, RNG_MT19937, seed & 0xFFFFFFFF, None, 0,
                          draft_catchup), None

    def generate_speculative(self, prompts, max_new_tokens: int, lookahead: int = 4, temperature: float = 1.0,
                             top_k: int = 0, top_p: float = 1.0, seed: int = 42,
                             uniforms: Optional[np.ndarray] = None,
                             draft_catchup: int = CATCHUP_REF) -> Tuple[np.ndarray, np.ndarray]:
        """prompts [B, S] -> (tokens [B, S + max(1, max_new)], stats [B, 4])."""
        p = np.ascontiguousarray(np.atleast_2d(prompts), np.int32)
        B, S = p.shape
        prm, keep = self._params(max_new_tokens, lookahead, temperature, top_k, top_p, seed, uniforms, draft_catchup)
        out = np.zeros((B, S + max(1, max_new_tokens)), np.int32)
        stats = np.zeros((B, 4), np.int64)
        self._check(self._lib.specdec_generate(self.h, C.byref(prm), p.ctypes.data, B, S, out.ctypes.data,
                                               stats.ctypes.data))
        del keep
        return out.astype(np.int64), stats

    # -- round-level session (specdec_prefill / specdec_step) ---------------
    def prefill(self, prompts, max_new_tokens: int, lookahead: int = 4, temperature: float = 1.0, top_k: int = 0,
                top_p: float = 1.0, seed: int = 42, uniforms: Optional[np.ndarray] = None,
                draft_catchup: int = CATCHUP_REF) -> None:
        """Opens a session: prefill of target and draft and the first token for
        prompts [B, S] (generate_speculative up to its round loop)."""
        p = np.ascontiguousarray(np.atleast_2d(prompts), np.int32)
        B, S = p.shape
        prm, keep = self._params(max_new_tokens, lookahead, temperature, top_k, top_p, seed, uniforms, draft_catchup)
        self._session = (B, S, lookahead, max_new_tokens)
        self._check(self._lib.specdec_prefill(self.h, C.byref(prm), p.ctypes.data, B, S))
        del keep

    def prefill_device(self, d_prompts: int, B: int, S: int, max_new_tokens: int, lookahead: int = 4,
                       temperature: float = 1.0, seed: int = 42, uniforms=None,
                       draft_catchup: int = CATCHUP_REF) -> None:
        """Device-pointer variant of prefill, enqueued on `stream`."""
        prm, keep = self._params(max_new_tokens, lookahead, temperature, 0, 1.0, seed, uniforms, draft_catchup)
        self._session = (B, S, lookahead, max_new_tokens)
        self._check(self._lib.specdec_prefill_device(self.h, C.byref(prm), C.c_void_p(d_prompts), B, S))
        del keep

    def step(self, rounds: int = 1, uniforms: Optional[np.ndarray] = None):
        """Up to `rounds` speculative rounds; returns (tokens [B, rounds*(k+1)],
        counts [B]): request b emitted tokens[b, :counts[b]] in this call.
        `uniforms` [B, rounds, 2k+1] replace the session table's rows of these rounds."""
        B, _, k, _ = self._session
        out = np.zeros((B, rounds * (k + 1)), np.int32)
        cnt = np.zeros(B, np.int32)
        u = None if uniforms is None else np.ascontiguousarray(uniforms, np.float32)
        self._check(self._lib.specdec_step(self.h, rounds, None if u is None else u.ctypes.data, out.ctypes.data,
                                           cnt.ctypes.data))
        return out, cnt

    def step_device(self, rounds: int, d_out: int, d_counts: int, cap: int, uniforms_ptr: int = 0) -> None:
        """Device-pointer variant of step (d_out [B][cap] int32, d_counts [B] int32),
        enqueued on `stream`; uniforms_ptr is a host or device [B][rounds][2k+1] table or 0."""
        self._check(self._lib.specdec_step_device(self.h, rounds, C.c_void_p(uniforms_ptr or None),
                                                  C.c_void_p(d_out), C.c_void_p(d_counts), cap))

    def session_tokens(self) -> Tuple[np.ndarray, np.ndarray]:
        """The open session's sequences [B, S + max(1, max_new)] and stats [B, 4]."""
        B, S, _, max_new = self._session
        out = np.zeros((B, S + max(1, max_new)), np.int32)
        stats = np.zeros((B, 4), np.int64)
        self._check(self._lib.specdec_session_tokens(self.h, out.ctypes.data, stats.ctypes.data))
        return out.astype(np.int64), stats

    def generate_tree(self, prompts, max_new_tokens: int, branching, temperature: float = 1.0, top_k: int = 0,
                      top_p: float = 1.0, seed: int = 42,
                      uniforms: Optional[np.ndarray] = None) -> Tuple[np.ndarray, np.ndarray]:
        """Tree speculation (specdec_generate_tree): branching = children per level,
        e.g. (4, 3, 2, 1).  Host uniforms: [B][rounds][depth * max(branching) + 1].
        Returns (tokens [B, S + max(1, max_new)], stats [B, 4])."""
        p = np.ascontiguousarray(np.atleast_2d(prompts), np.int32)
        B, S = p.shape
        prm, keep = self._params(max_new_tokens, 1, temperature, top_k, top_p, seed, uniforms, CATCHUP_CORRECT)
        br = list(branching)
        tree = _Tree(len(br), (C.c_int32 * 8)(*br))
        out = np.zeros((B, S + max(1, max_new_tokens)), np.int32)
        stats = np.zeros((B, 4), np.int64)
        self._check(self._lib.specdec_generate_tree(self.h, C.byref(prm), C.byref(tree), p.ctypes.data, B, S,
                                                    out.ctypes.data, stats.ctypes.data))
        del keep
        return out.astype(np.int64), stats

    def generate_tree_device(self, d_prompts: int, B: int, S: int, d_out: int, d_stats: int, max_new_tokens: int,
                             branching, temperature: float = 1.0, seed: int = 42, uniforms=None) -> None:
        """Device-pointer variant of generate_tree, enqueued on `stream`."""
        prm, keep = self._params(max_new_tokens, 1, temperature, 0, 1.0, seed, uniforms, CATCHUP_CORRECT)
        br = list(branching)
        tree = _Tree(len(br), (C.c_int32 * 8)(*br))
        self._check(self._lib.specdec_generate_tree_device(self.h, C.byref(prm), C.byref(tree), C.c_void_p(d_prompts),
                                                           B, S, C.c_void_p(d_out), C.c_void_p(d_stats)))
        del keep

    def generate_device(self, d_prompts: int, B: int, S: int, d_out: int, d_stats: int, max_new_tokens: int,
                        lookahead: int = 4, temperature: float = 1.0, seed: int = 42, uniforms=None,
                        draft_catchup: int = CATCHUP_REF) -> None:
        """Device-pointer variant (ints are raw CUDA pointers); enqueued on `stream`."""
        prm, keep = self._params(max_new_tokens, lookahead, temperature, 0, 1.0, seed, uniforms, draft_catchup)
        self._check(self._lib.specdec_generate_device(self.h, C.byref(prm), C.c_void_p(d_prompts), B, S,
                                                      C.c_void_p(d_out), C.c_void_p(d_stats)))
        del keep

    def generate_advanced(self, prompts, max_new_tokens: int, temperature: float = 1.0, top_k: int = 0,
                          top_p: float = 1.0, seed: int = 42,
                          uniforms: Optional[np.ndarray] = None) -> Tuple[np.ndarray, np.ndarray]:
        """Autoregressive decoding with the target's KV cache, as the reference's
        ``generate_advanced(prompt, max_new_tokens, temperature, top_k, top_p,
        seed, use_kv_cache=true)`` (src/nn/layer.cpp:1239-1380), over B requests
        (request b draws from mt19937(seed + b), or from uniforms[b][step][0]).
        prompts [B, S] -> (tokens [B, S + max_new], stats [B, 4] = steps, 0, 0, 0)."""
        p = np.ascontiguousarray(np.atleast_2d(prompts), np.int32)
        B, S = p.shape
        prm, keep = self._params(max_new_tokens, 1, temperature, top_k, top_p, seed, uniforms, CATCHUP_REF)
        out = np.zeros((B, S + max_new_tokens), np.int32)
        stats = np.zeros((B, 4), np.int64)
        self._check(self._lib.specdec_generate_ar(self.h, C.byref(prm), p.ctypes.data, B, S, out.ctypes.data,
                                                  stats.ctypes.data))
        del keep
        return out.astype(np.int64), stats

    def generate_advanced_device(self, d_prompts: int, B: int, S: int, d_out: int, d_stats: int,
                                 max_new_tokens: int, temperature: float = 1.0, seed: int = 42,
                                 uniforms=None) -> None:
        """Device-pointer variant of generate_advanced, enqueued on `stream`
        (d_out [B][S + max(1, max_new)])."""
        prm, keep = self._params(max_new_tokens, 1, temperature, 0, 1.0, seed, uniforms, CATCHUP_REF)
        self._check(self._lib.specdec_generate_ar_device(self.h, C.byref(prm), C.c_void_p(d_prompts), B, S,
                                                         C.c_void_p(d_out), C.c_void_p(d_stats)))
        del keep

    def forward_logits(self, role: int, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, np.int32).ravel()
        V = self.target.vocab
        out = np.zeros((t.size, V), np.float32)
        self._check(self._lib.specdec_forward_logits(self.h, role, t.ctypes.data, t.size, out.ctypes.data))
        return out

    def forward_logits_noalloc(self, role: int, d_tokens: int, S: int, d_logits: int, stream: int = 0,
                               d_status: int = 0) -> None:
        """Device-buffer forward that allocates nothing (see include/specdec.h).

        For callers that may not allocate device memory at call time; all
        working memory comes from the library's fixed 8 MiB device array, so
        overlapping calls on one device must be serialised by the caller.
        d_status (a device int32, optional) receives the device-side error bits."""
        self._check(self._lib.specdec_forward_logits_noalloc(self.h, role, C.c_void_p(d_tokens), S,
                                                             C.c_void_p(d_logits), C.c_void_p(stream or None),
                                                             C.c_void_p(d_status or None)))

    @property
    def stream(self) -> int:
        return int(self._lib.specdec_stream(self.h) or 0)

    def last_launch_count(self) -> int:
        return int(self._lib.specdec_last_launch_count(self.h))

    def time_linear(self, role: int, layer: int, which: int, rows: int, reps: int, flush_ptr: int = 0,
                    flush_bytes: int = 0):
        """Mean device time (us) of one linear layer's kernel over `rows` rows, each
        launch alone with the L2 flushed before it, and its algorithmic bytes."""
        us, nb = C.c_float(0.0), C.c_double(0.0)
        self._check(self._lib.specdec_time_linear(self.h, role, layer, which, rows, reps, C.c_void_p(flush_ptr),
                                                  C.c_size_t(flush_bytes), C.byref(us), C.byref(nb)))
        return float(us.value), float(nb.value)

    def time_attention(self, role: int, layer: int, q_per_req: int, reps: int, flush_ptr: int = 0,
                       flush_bytes: int = 0):
        """Mean device time (us) of one layer's attention launch over the open
        session's caches (q_per_req rows per request), each launch alone with
        the L2 flushed before it, and its algorithmic bytes."""
        us, nb = C.c_float(0.0), C.c_double(0.0)
        self._check(self._lib.specdec_time_attention(self.h, role, layer, q_per_req, reps, C.c_void_p(flush_ptr),
                                                     C.c_size_t(flush_bytes), C.byref(us), C.byref(nb)))
        return float(us.value), float(nb.value)
