"""swiftlet_b200 — B200 (sm_100a) decode backend for Qwen3-Next / Qwen3.5-MoE.

Python mirror of Swiftlet's model API over the C ABI in
``include/swiftlet_cuda.h`` (``libswiftlet_cuda.so``, built in-tree):

* ``QwenCUDAModel(model_dir, cache_budget_gb=0)`` — QwenMetalModel
  (Sources/SwiftletCore/QwenMetalModel.swift:104) with ``config``,
  ``model_dir``, ``step(tokens, state)``, ``expert_cache`` and
  ``shrink_cache(to_gb)``.
* ``DecodeState`` — QwenCPUModel.DecodeState (QwenCPUModel.swift:183).
* ``TextGenerator`` — greedy generation loop (TextGenerator.swift:19-98).

There is no CPU fallback: without the CUDA library or a GPU every call
raises ``SwiftletError``.
"""
from __future__ import annotations

import ctypes as C
import json
import os
import weakref
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libswiftlet_cuda.so")

SWL_OK = 0
SWL_ERR_INVALID = -1
SWL_ERR_IO = -2
SWL_ERR_FORMAT = -3
SWL_ERR_CUDA = -4
SWL_ERR_OOM = -5
SWL_ERR_UNSUPPORTED = -6
SWL_ERR_CAPACITY = -7


class SwiftletError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code


class swl_config(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "hidden_size", "num_hidden_layers", "num_attention_heads", "num_key_value_heads", "head_dim",
        "vocab_size", "full_attention_interval", "linear_num_value_heads", "linear_num_key_heads",
        "linear_key_head_dim", "linear_value_head_dim", "linear_conv_kernel_dim", "num_experts",
        "num_experts_per_tok", "moe_intermediate_size", "shared_expert_intermediate_size", "norm_topk_prob",
        "tie_word_embeddings", "split_delta_layout", "rotary_dims")] + [
        ("rope_theta", C.c_double), ("partial_rotary_factor", C.c_double), ("rms_norm_eps", C.c_double)]


class swl_verify_report(C.Structure):
    _fields_ = [("checked", C.c_int64), ("ok", C.c_int64), ("corrupt", C.c_int64), ("missing", C.c_int64),
                ("first_bad", C.c_char * 256)]


class swl_affine_matrix(C.Structure):
    """A device-resident MLX-affine matrix (see include/swiftlet_cuda.h)."""
    _fields_ = [("weight", C.c_void_p), ("scales", C.c_void_p), ("biases", C.c_void_p), ("rows", C.c_int32),
                ("cols", C.c_int32), ("bits", C.c_int32), ("group", C.c_int32), ("scale_dtype", C.c_int32)]


class swl_pool_info(C.Structure):
    _fields_ = [(n, C.c_int64) for n in (
        "expert_stride", "slot_count", "allocated_slots", "hits", "misses", "resident_bytes")]


# Every entry point of include/swiftlet_cuda.h with its ctypes signature.
_P, _I, _I64, _D = C.c_void_p, C.c_int, C.c_int64, C.c_double
_SIGNATURES = {
    "swl_last_error": (C.c_char_p, []),
    "swl_model_open": (_I, [C.c_char_p, _D, _I, C.POINTER(_P)]),
    "swl_model_close": (_I, [_P]),
    "swl_model_config": (_I, [_P, C.POINTER(swl_config)]),
    "swl_state_new": (_I, [_P, C.c_int32, C.POINTER(_P)]),
    "swl_state_free": (_I, [_P]),
    "swl_state_position": (C.c_int32, [_P]),
    "swl_step": (_I, [_P, _P, _P, C.c_int32, _P]),
    "swl_step_batch": (_I, [_P, _P, _P, _P, C.c_int32, _P]),
    "swl_step_device": (_I, [_P, _P, _P, C.c_int32, _P, _P]),
    "swl_step_batch_device": (_I, [_P, _P, C.c_int32, _P, _P, _P]),
    "swl_batch_supported": (_I, [_P, C.c_char_p, C.c_int32]),
    "swl_sample_device": (_I, [_P, C.c_int32, C.c_int32, _I64, _P, _P, C.c_int32, _P, C.c_int32, _P, _P,
                               C.c_int32, _P, _P, _P]),
    "swl_ep_unique_id": (_I, [_P, C.c_int32]),
    "swl_ep_init": (_I, [_P, C.c_int32, C.c_int32, _P, C.c_int32, C.c_int32]),
    "swl_ep_info": (_I, [_P] * 5),
    "swl_ep_timing": (_I, [_P, C.c_int32, C.POINTER(C.c_double)]),
    "swl_pool_stats": (_I, [_P, C.POINTER(swl_pool_info)]),
    "swl_pool_resize": (_I, [_P, _D]),
    "swl_set_stream": (_I, [_P, _P]),
    "swl_debug_dequant": (_I, [_P, C.c_char_p, _I64, _I64, _P]),
    "swl_debug_tensor_bytes": (_I, [_P, C.c_char_p, _I64, _I64, _P, _I64]),
    "swl_debug_layer": (_I, [_P, _P, C.c_int32, _P, _P, _P, _P]),
    "swl_debug_delta_state": (_I, [_P, _P, C.c_int32, _P]),
    "swl_debug_kernel_path": (_I, [_P, C.c_char_p, C.c_int32]),
    "swl_state_reset": (_I, [_P]),
    "swl_ep_set_liveness": (_I, [_P, _P, _P]),
    "swl_kernel_gated_delta": (_I, [_P] * 7 + [C.c_int32] * 5),
    "swl_bench_gated_delta": (_I, [C.c_int32] * 6 + [C.POINTER(C.c_float), C.POINTER(C.c_double)]),
    "swl_bench_moe_sweep": (_I, [_P, C.c_int32, C.c_int32, C.POINTER(C.c_float), C.POINTER(C.c_double),
                                 C.POINTER(C.c_int32), C.POINTER(C.c_int32)]),
    "swl_bench_delta_sweep": (_I, [_P, C.c_int32, C.c_int32, C.POINTER(C.c_float), C.POINTER(C.c_double),
                                   C.POINTER(C.c_int32)]),
    "swl_qpack_verify": (_I, [C.c_char_p, C.c_char_p, C.c_int32, C.POINTER(swl_verify_report)]),
    "swl_sha256_file": (_I, [C.c_char_p, C.c_char_p]),
    "swl_state_copy": (_I, [_P, _P]),
    "swl_state_save": (_I, [_P, _P, C.c_int64, C.POINTER(C.c_int64)]),
    "swl_state_load": (_I, [_P, _P, C.c_int64]),
    "swl_debug_wait_timeout": (_I, [_P, C.c_int32]),
    "swl_bench_expert_sweep": (_I, [_P, C.c_int32, _P, _P, _P]),
    "swl_trace_dump": (_I, [_P, C.c_char_p]),
    "swl_kernel_gemv_affine": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _P, _P]),
    "swl_kernel_expert_swiglu": (_I, [_P] * 9 + [_I, _I, _I, _I, _I, _P, _P]),
    "swl_expert_swiglu_noalloc": (_I, [C.POINTER(swl_affine_matrix)] * 3 + [_P, _P, _P, _P]),
}

_lib = None


def library_path() -> str:
    return LIB_PATH


def lib():
    """Loads libswiftlet_cuda.so (building it first when sources are newer)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            from . import build as _build
            _build.build()
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _check(rc: int) -> None:
    if rc != SWL_OK:
        raise SwiftletError(rc, lib().swl_last_error().decode(errors="replace"))


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


@dataclass
class QwenConfig:
    """Fields of QwenConfig (Sources/SwiftletCore/QwenConfig.swift:10-50)."""
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    vocab_size: int
    full_attention_interval: int
    linear_num_value_heads: int
    linear_num_key_heads: int
    linear_key_head_dim: int
    linear_value_head_dim: int
    linear_conv_kernel_dim: int
    num_experts: int
    num_experts_per_tok: int
    moe_intermediate_size: int
    shared_expert_intermediate_size: int
    norm_topk_prob: bool
    tie_word_embeddings: bool
    split_delta_layout: bool
    rotary_dims: int
    rope_theta: float
    partial_rotary_factor: float
    rms_norm_eps: float

    def is_linear_layer(self, i: int) -> bool:
        """QwenConfig.isLinearLayer (QwenConfig.swift:108-110)."""
        return (i + 1) % self.full_attention_interval != 0

    @property
    def key_dim(self) -> int:
        return self.linear_num_key_heads * self.linear_key_head_dim

    @property
    def value_dim(self) -> int:
        return self.linear_num_value_heads * self.linear_value_head_dim


@dataclass
class ExpertCacheStats:
    """ExpertCache counters (ExpertCache.swift:11,21-22,40-41)."""
    stride: int
    slot_count: int
    allocated_slots: int
    hits: int
    misses: int
    resident_bytes: int


class DecodeState:
    """Per-sequence device state (QwenCPUModel.DecodeState). Created by
    ``QwenCUDAModel.new_state`` or lazily on the first ``step``."""

    def __init__(self, max_ctx: int = 4096):
        self.max_ctx = int(max_ctx)
        self._h = None
        self._model = None

    def _bind(self, model: "QwenCUDAModel") -> int:
        if self._h is None:
            h = C.c_void_p()
            _check(lib().swl_state_new(model._h, self.max_ctx, C.byref(h)))
            self._h = h.value
            self._model = model
            model._states.append(weakref.ref(self))
        elif self._model is not model:
            raise SwiftletError(SWL_ERR_INVALID, "state belongs to another model")
        return self._h

    @property
    def position(self) -> int:
        return 0 if self._h is None else lib().swl_state_position(self._h)

    def free(self) -> None:
        if self._h is not None:
            lib().swl_state_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class QwenCUDAModel:
    """Drop-in for QwenMetalModel: ``step(tokens, state) -> logits``."""

    def __init__(self, model_dir: str, cache_budget_gb: float = 0.0, device: int = 0):
        h = C.c_void_p()
        _check(lib().swl_model_open(os.fsencode(model_dir), float(cache_budget_gb), int(device), C.byref(h)))
        self._h = h.value
        self.model_dir = model_dir
        cfg = swl_config()
        _check(lib().swl_model_config(self._h, C.byref(cfg)))
        vals = {name: getattr(cfg, name) for name, _ in swl_config._fields_}
        for b in ("norm_topk_prob", "tie_word_embeddings", "split_delta_layout"):
            vals[b] = bool(vals[b])
        self.config = QwenConfig(**vals)
        self._states: list = []

    def close(self) -> None:
        if getattr(self, "_h", None):
            for ref in self._states:   # device states must go before the model
                st = ref()
                if st is not None:
                    st.free()
            lib().swl_model_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def new_state(self, max_ctx: int = 4096) -> DecodeState:
        s = DecodeState(max_ctx)
        s._bind(self)
        return s

    def step(self, tokens, state: DecodeState) -> np.ndarray:
        """InferenceModel.step (TextGenerator.swift:7): consumes the tokens,
        advances ``state.position`` and returns the last position's logits."""
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32).reshape(-1))
        out = np.empty(self.config.vocab_size, np.float32)
        _check(lib().swl_step(self._h, state._bind(self), _ptr(t), len(t), _ptr(out)))
        return out

    def step_batch(self, token_lists, states) -> np.ndarray:
        counts = np.array([len(t) for t in token_lists], np.int32)
        flat = np.ascontiguousarray(np.concatenate([np.asarray(t, np.int32).reshape(-1) for t in token_lists]))
        handles = (C.c_void_p * len(states))(*[s._bind(self) for s in states])
        out = np.empty((len(states), self.config.vocab_size), np.float32)
        _check(lib().swl_step_batch(self._h, handles, _ptr(flat), _ptr(counts), len(states), _ptr(out)))
        return out

    def step_batch_device(self, states, d_tokens: int, d_logits: int = 0, d_greedy: int = 0) -> None:
        """One token for each state, device-resident tokens / logits / greedy ids."""
        handles = (C.c_void_p * len(states))(*[s._bind(self) for s in states])
        _check(lib().swl_step_batch_device(self._h, handles, len(states), C.c_void_p(d_tokens),
                                           C.c_void_p(d_logits or None), C.c_void_p(d_greedy or None)))

    def batch_supported(self) -> tuple[bool, str]:
        """Whether step_batch runs the batched kernels for this model (and why not)."""
        buf = C.create_string_buffer(256)
        rc = lib().swl_batch_supported(self._h, buf, 256)
        if rc < 0:
            _check(rc)
        return rc == 1, buf.value.decode()

    def ep_init(self, rank: int, world: int, ep_id: bytes, tokens_per_rank: int) -> None:
        """Joins an expert-parallel group of `world` ranks (swl_ep_init); every
        rank passes the same id (from ep_unique_id) and tokens_per_rank."""
        if len(ep_id) != EP_ID_BYTES:
            raise ValueError(f"expert-parallel id must be {EP_ID_BYTES} bytes")
        buf = C.create_string_buffer(bytes(ep_id), EP_ID_BYTES)
        _check(lib().swl_ep_init(self._h, int(rank), int(world), C.cast(buf, C.c_void_p), EP_ID_BYTES,
                                 int(tokens_per_rank)))

    def ep_info(self) -> tuple[bool, int, int, int, int]:
        """(on, rank, world, first owned expert, end of the owned range)."""
        v = [C.c_int32() for _ in range(4)]
        rc = lib().swl_ep_info(self._h, *[C.byref(x) for x in v])
        if rc < 0:
            _check(rc)
        return (rc == 1, *[x.value for x in v])

    def ep_timing(self, reset: bool = False) -> dict | None:
        """Collective timing of expert-parallel steps (swl_ep_timing), or None
        when inactive (it needs SWL_EP_TIMING=1 and SWL_EP_NO_GRAPH=1 set
        before ep_init)."""
        out = (C.c_double * 4)()
        rc = lib().swl_ep_timing(self._h, int(reset), out)
        if rc < 0:
            _check(rc)
        if rc != 1:
            return None
        return {"steps": int(out[0]), "step_ms": out[1], "collectives": int(out[2]), "collective_ms": out[3]}

    def step_device(self, d_tokens: int, n: int, state: DecodeState, d_logits: int = 0, d_greedy: int = 0) -> None:
        """Device-pointer form (tokens/logits already in HBM)."""
        _check(lib().swl_step_device(self._h, state._bind(self), C.c_void_p(d_tokens), int(n),
                                     C.c_void_p(d_logits or None), C.c_void_p(d_greedy or None)))

    def ep_set_liveness(self, callback) -> None:
        """swl_ep_set_liveness: callback(step) -> True while every peer is
        alive and at `step` (None removes it)."""
        if callback is None:
            self._liveness = None
            _check(lib().swl_ep_set_liveness(self._h, None, None))
            return
        fn = _LIVENESS_FN(lambda ctx, step: 0 if callback(int(step)) else 1)
        self._liveness = fn  # keep the C callback alive
        _check(lib().swl_ep_set_liveness(self._h, C.cast(fn, C.c_void_p), None))

    def set_stream(self, cuda_stream: int | None) -> None:
        _check(lib().swl_set_stream(self._h, C.c_void_p(cuda_stream or None)))

    @property
    def expert_cache(self) -> ExpertCacheStats:
        p = swl_pool_info()
        _check(lib().swl_pool_stats(self._h, C.byref(p)))
        return ExpertCacheStats(p.expert_stride, p.slot_count, p.allocated_slots, p.hits, p.misses, p.resident_bytes)

    def shrink_cache(self, to_gb: float) -> None:
        """QwenMetalModel.shrinkCache(toGB:) (QwenMetalModel.swift:324)."""
        _check(lib().swl_pool_resize(self._h, float(to_gb)))

    # -- inspection (parity tests) -------------------------------------
    def debug_dequant(self, module: str, r0: int, r1: int, cols: int) -> np.ndarray:
        out = np.empty((r1 - r0, cols), np.float32)
        _check(lib().swl_debug_dequant(self._h, module.encode(), r0, r1, _ptr(out)))
        return out

    def debug_tensor_bytes(self, name: str, e0: int, e1: int, elem_bytes: int) -> bytes:
        buf = C.create_string_buffer(max(1, (e1 - e0) * elem_bytes))
        _check(lib().swl_debug_tensor_bytes(self._h, name.encode(), e0, e1, buf, (e1 - e0) * elem_bytes))
        return buf.raw[: (e1 - e0) * elem_bytes]

    def debug_layer(self, state: DecodeState, layer: int, h):
        h = np.ascontiguousarray(h, dtype=np.float32).reshape(-1)
        out = np.empty_like(h)
        k = self.config.num_experts_per_tok
        ids = np.empty(k, np.int32)
        w = np.empty(k, np.float32)
        _check(lib().swl_debug_layer(self._h, state._bind(self), layer, _ptr(h), _ptr(out), _ptr(ids), _ptr(w)))
        return out, ids, w

    def bench_expert_sweep(self, iters: int):
        """(elapsed ms, algorithmic bytes per layer, launches) of `iters` expert sweeps."""
        ms = C.c_float()
        b = C.c_double()
        n = C.c_int32()
        _check(lib().swl_bench_expert_sweep(self._h, int(iters), C.byref(ms), C.byref(b), C.byref(n)))
        return ms.value, b.value, n.value

    def bench_moe_sweep(self, T: int, iters: int):
        """(ms, bytes per sweep, distinct experts per sweep, launches) of the batched MoE block."""
        ms, b, u, n = C.c_float(), C.c_double(), C.c_int32(), C.c_int32()
        _check(lib().swl_bench_moe_sweep(self._h, int(T), int(iters), C.byref(ms), C.byref(b), C.byref(u),
                                         C.byref(n)))
        return ms.value, b.value, u.value, n.value

    def bench_delta_sweep(self, T: int, iters: int):
        """(ms, bytes per sweep, launches) of the DeltaNet decode step over every DeltaNet layer."""
        ms, b, n = C.c_float(), C.c_double(), C.c_int32()
        _check(lib().swl_bench_delta_sweep(self._h, int(T), int(iters), C.byref(ms), C.byref(b), C.byref(n)))
        return ms.value, b.value, n.value

    def trace_dump(self, path: str) -> None:
        """Writes the per-block kernel timeline (needs SWL_TRACE at open)."""
        _check(lib().swl_trace_dump(self._h, path.encode()))

    def debug_delta_state(self, state: DecodeState, layer: int) -> np.ndarray:
        c = self.config
        out = np.empty((c.linear_num_value_heads, c.linear_value_head_dim, c.linear_key_head_dim), np.float32)
        _check(lib().swl_debug_delta_state(self._h, state._bind(self), layer, _ptr(out)))
        return out

    # ---- conversation-state reuse (SwiftletSession.swift:114-132, 193-213) ----
    def reset_state(self, state: DecodeState) -> None:
        """SwiftletSession.resetConversation: position 0, zeroed recurrent state."""
        _check(lib().swl_state_reset(state._bind(self)))

    def copy_state(self, dst: DecodeState, src: DecodeState) -> None:
        """Forks `src` into `dst` (position, conv rings, delta states, KV rows)."""
        _check(lib().swl_state_copy(dst._bind(self), src._bind(self)))

    def save_state(self, state: DecodeState) -> bytes:
        """Host snapshot of the state's whole decode state."""
        h = state._bind(self)
        n = C.c_int64()
        _check(lib().swl_state_save(h, None, 0, C.byref(n)))
        buf = C.create_string_buffer(n.value)
        _check(lib().swl_state_save(h, buf, n.value, C.byref(n)))
        return buf.raw[:n.value]

    def load_state(self, state: DecodeState, data: bytes) -> None:
        """Restores a snapshot taken by save_state on a model of the same shape."""
        _check(lib().swl_state_load(state._bind(self), data, len(data)))

    def kernel_path(self) -> list[str]:
        """Kernel family of every launch of one single-token decode step
        (``swl_debug_kernel_path``): e.g. ``["embed", "igemv", "delta", ...]``."""
        buf = C.create_string_buffer(1 << 16)
        _check(lib().swl_debug_kernel_path(self._h, buf, len(buf)))
        return buf.value.decode().split(",")

    def debug_wait_timeout(self, limit_us: int) -> None:
        """One bounded wait that nothing completes (``swl_debug_wait_timeout``):
        raises SwiftletError(SWL_ERR_CUDA) once it has given up."""
        _check(lib().swl_debug_wait_timeout(self._h, int(limit_us)))


class swl_sample_options(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("presence_penalty", C.c_float),
                ("frequency_penalty", C.c_float), ("top_k", C.c_int32)]


def sample_device(d_logits: int, nseq: int, vocab: int, row_stride: int, *, temperature: float = 0.7,
                  top_k: int = 20, top_p: float = 0.8, presence_penalty: float = 0.0, frequency_penalty: float = 0.0,
                  d_suppress: int = 0, n_suppress: int = 0, d_eos: int = 0, n_eos: int = 0, d_ban_eos: int = 0,
                  d_counts: int = 0, update_counts: bool = False, d_uniform: int = 0, d_out: int = 0,
                  stream: int = 0) -> None:
    """SwiftletSession.sample on the GPU for nseq device rows (swl_sample_device);
    the defaults are GenerationOptions' (SwiftletSession.swift:20-28) without penalties."""
    o = swl_sample_options(float(temperature), float(top_p), float(presence_penalty), float(frequency_penalty),
                           int(top_k))
    v = lambda p: C.c_void_p(p or None)  # noqa: E731
    _check(lib().swl_sample_device(v(d_logits), int(nseq), int(vocab), int(row_stride), C.byref(o), v(d_suppress),
                                   int(n_suppress), v(d_eos), int(n_eos), v(d_ban_eos), v(d_counts),
                                   int(bool(update_counts)), v(d_uniform), v(d_out), v(stream)))


EP_ID_BYTES = 128


def ep_unique_id() -> bytes:
    """A fresh expert-parallel communicator id (swl_ep_unique_id)."""
    buf = C.create_string_buffer(EP_ID_BYTES)
    _check(lib().swl_ep_unique_id(C.cast(buf, C.c_void_p), EP_ID_BYTES))
    return buf.raw


def ep_unique_id_broadcast(rank: int) -> bytes:
    """Rank 0 makes the id and torch.distributed (already initialised, any
    backend) hands it to the other ranks."""
    import torch.distributed as dist
    box = [ep_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    return box[0]


def gemv_affine(packed, scales, biases, out_dim: int, in_dim: int, group: int, bits: int, x) -> np.ndarray:
    """One MLX-affine GEMV on the GPU (the fast kernel of the decode path)."""
    packed = np.ascontiguousarray(packed, dtype=np.uint32)
    sd = {np.dtype(np.float32): 0, np.dtype(np.uint16): 1, np.dtype(np.float16): 2}[np.asarray(scales).dtype]
    scales = np.ascontiguousarray(scales)
    biases = np.ascontiguousarray(biases)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(out_dim, np.float32)
    _check(lib().swl_kernel_gemv_affine(_ptr(packed), _ptr(scales), _ptr(biases), sd, out_dim, in_dim, group, bits,
                                        _ptr(x), _ptr(y)))
    return y


def expert_swiglu(gate, up, down, hidden: int, inter: int, group: int, bits: int, x) -> np.ndarray:
    """One expert's SwiGLU on the GPU; each matrix is (packed uint32, scales, biases)."""
    arrs = [np.ascontiguousarray(a) for m in (gate, up, down) for a in m]
    sd = {np.dtype(np.float32): 0, np.dtype(np.uint16): 1, np.dtype(np.float16): 2}[arrs[1].dtype]
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(hidden, np.float32)
    _check(lib().swl_kernel_expert_swiglu(*[_ptr(a) for a in arrs], sd, bits, group, hidden, inter, _ptr(x), _ptr(y)))
    return y


def gated_delta(q, k, v, g, beta, state, T, Hk, Hv, Dk, Dv):
    """Gated delta rule over T steps on the GPU's chunked prompt kernel. Returns (y, state)."""
    arrs = [np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v, g, beta)]
    st = np.array(state, dtype=np.float32, copy=True)
    y = np.zeros(T * Hv * Dv, np.float32)
    _check(lib().swl_kernel_gated_delta(*[_ptr(a) for a in arrs], _ptr(st), _ptr(y), T, Hk, Hv, Dk, Dv))
    return y, st


def bench_gated_delta(T, Hk, Hv, Dk, Dv, iters):
    """(ms, flops) of `iters` launches of the chunked prompt delta-rule kernel over T tokens."""
    ms, fl = C.c_float(), C.c_double()
    _check(lib().swl_bench_gated_delta(T, Hk, Hv, Dk, Dv, iters, C.byref(ms), C.byref(fl)))
    return ms.value, fl.value


_LIVENESS_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int32)


def ep_store_liveness(store, rank: int, world: int, timeout_s: float = 30.0):
    """A liveness callback for ep_set_liveness over a torch.distributed store:
    at each step a rank publishes the step it is entering, then waits (up to
    timeout_s) until every peer has published it too; False when one does
    not, i.e. it left or stopped."""
    import time

    def alive(step: int) -> bool:
        store.set(f"swl_ep/{rank}", str(step))
        deadline = time.monotonic() + timeout_s
        for p in range(world):
            if p == rank:
                continue
            while True:
                try:
                    seen = int(store.get(f"swl_ep/{p}"))
                except Exception:
                    seen = -1
                if seen >= step:
                    break
                if time.monotonic() > deadline:
                    return False
                time.sleep(0.002)
        return True

    return alive


def verify_container(container: str, hashes_json: str | None = None, delete_corrupt: bool = False) -> dict:
    """SHA-256 check of a .qpack container against its hashes.json
    (scripts/verify_container.py). Returns the counts; raises SwiftletError
    (SWL_ERR_FORMAT) when a file is corrupt or missing, after filling them."""
    r = swl_verify_report()
    rc = lib().swl_qpack_verify(os.fsencode(container), os.fsencode(hashes_json) if hashes_json else None,
                                int(bool(delete_corrupt)), C.byref(r))
    rep = {"checked": r.checked, "ok": r.ok, "corrupt": r.corrupt, "missing": r.missing,
           "first_bad": r.first_bad.decode()}
    if rc != SWL_OK:
        err = SwiftletError(rc, lib().swl_last_error().decode())
        err.report = rep
        raise err
    return rep


def sha256_file(path: str) -> str:
    out = C.create_string_buffer(65)
    _check(lib().swl_sha256_file(os.fsencode(path), out))
    return out.value.decode()


def expert_swiglu_noalloc(gate: swl_affine_matrix, up: swl_affine_matrix, down: swl_affine_matrix, d_x: int,
                          d_y: int, stream: int | None = None, d_status: int | None = None) -> None:
    """Allocation-free expert SwiGLU on device buffers (queued on `stream`, not waited for).
    `d_status` (device int32 address, optional) gets bit 0 set when a bounded
    wait inside the kernels gave up."""
    _check(lib().swl_expert_swiglu_noalloc(C.byref(gate), C.byref(up), C.byref(down), C.c_void_p(d_x),
                                           C.c_void_p(d_y), C.c_void_p(d_status or None),
                                           C.c_void_p(stream or None)))


class TextGenerator:
    """Engine-agnostic greedy loop (TextGenerator.swift:19-98)."""

    def __init__(self, model):
        self.model = model
        self.eos_tokens = self.eos_token_ids(model.model_dir)

    @staticmethod
    def eos_token_ids(model_dir: str) -> set[int]:
        """EOS ids from generation_config.json / config.json (TextGenerator.swift:29-38)."""
        eos: set[int] = set()
        for name in ("generation_config.json", "config.json"):
            p = os.path.join(model_dir, name)
            try:
                obj = json.load(open(p))
            except (OSError, ValueError):
                continue
            v = obj.get("eos_token_id")
            if isinstance(v, int):
                eos.add(v)
            elif isinstance(v, list):
                eos.update(x for x in v if isinstance(x, int))
        return eos

    def generate(self, prompt_ids, max_new: int, on_token=lambda t: True, state: DecodeState | None = None) -> dict:
        """Greedy decode; EOS stops generation and is not reported."""
        import time
        state = state if state is not None else DecodeState()
        stats = {"prompt_tokens": len(prompt_ids), "generated_tokens": 0}
        t0 = time.perf_counter()
        logits = self.model.step(list(prompt_ids), state)
        stats["prefill_seconds"] = time.perf_counter() - t0
        t1 = time.perf_counter()
        for _ in range(max_new):
            best = int(np.argmax(logits))   # first maximal index, as the reference's `>` scan
            if best in self.eos_tokens:
                break
            stats["generated_tokens"] += 1
            if not on_token(best):
                break
            logits = self.model.step([best], state)
        stats["decode_seconds"] = time.perf_counter() - t1
        return stats
