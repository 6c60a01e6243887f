"""CPU oracle for the Swiftlet decode path — TEST INFRASTRUCTURE ONLY.

ctypes wrapper over ``oracle/build/liboracle.so``, the C++ restatement of
Swiftlet's ``QwenCPUModel`` (Sources/SwiftletCore/QwenCPUModel.swift) and of
``Checkpoint`` / ``Safetensors`` / ``QwenConfig``. Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` import this package; the CUDA product never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "build", "liboracle.so")

_lib = None


def build() -> str:
    """Compile the oracle library (make, g++ -O3 -fopenmp)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        P, I, F, D = C.c_void_p, C.c_int, C.c_float, C.c_double
        fp = C.POINTER(C.c_float)
        ip = C.POINTER(C.c_int32)
        L.orc_last_error.restype = C.c_char_p
        L.orc_open.restype = P
        L.orc_open.argtypes = [C.c_char_p, I]
        L.orc_close.argtypes = [P]
        L.orc_config_int.argtypes = [P, C.c_char_p]
        L.orc_forward.argtypes = [P, ip, I, fp, fp, fp, fp, ip, ip]
        L.orc_layer_forward.argtypes = [P, fp, I, I, P, fp]
        L.orc_moe_forward.argtypes = [P, I, fp, I, fp, ip, fp, fp]
        L.orc_mixer_forward.argtypes = [P, I, fp, I, P, fp]
        L.orc_state_new.restype = P
        L.orc_state_free.argtypes = [P]
        L.orc_state_position.argtypes = [P]
        L.orc_state_advance.argtypes = [P, I]
        L.orc_state_delta.argtypes = [P, P, I, fp]
        L.orc_step.argtypes = [P, P, ip, I, fp]
        L.orc_route_gap.restype = C.c_double
        L.orc_route_gap.argtypes = [P, I]
        L.orc_dequant.argtypes = [P, C.c_char_p, C.c_int64, C.c_int64, fp]
        L.orc_tensor_bytes.argtypes = [P, C.c_char_p, C.c_int64, C.c_int64, P]
        L.orc_tensor_info.argtypes = [P, C.c_char_p, C.c_char_p, C.POINTER(C.c_int64)]
        L.orc_set_threads.argtypes = [I]
        L.orc_gemv_affine.argtypes = [C.POINTER(C.c_uint32), P, P, I, I, I, I, I, fp, fp]
        L.orc_gated_delta.argtypes = [fp, fp, fp, fp, fp, fp, fp, I, I, I, I, I]
        L.orc_expert_swiglu.argtypes = [P] * 9 + [I, I, I, I, I, fp, fp]
        _lib = L
    return _lib


def _f(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _i(a):
    return a.ctypes.data_as(C.POINTER(C.c_int32))


def _check(rc):
    if rc != 0:
        raise RuntimeError("oracle: " + lib().orc_last_error().decode())


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def max_threads() -> int:
    return lib().orc_max_threads()


class DecodeState:
    """Per-session state (QwenCPUModel.DecodeState, QwenCPUModel.swift:183-193)."""

    def __init__(self):
        self._h = lib().orc_state_new()

    def __del__(self):
        if getattr(self, "_h", None):
            lib().orc_state_free(self._h)
            self._h = None

    @property
    def position(self) -> int:
        return lib().orc_state_position(self._h)

    def advance(self, n: int) -> None:
        lib().orc_state_advance(self._h, int(n))


class OracleModel:
    """QwenCPUModel restated: ``forward``, ``step``, ``layer_forward``."""

    def __init__(self, model_dir: str, retain_all_layers: bool = True):
        self._h = lib().orc_open(model_dir.encode(), int(retain_all_layers))
        if not self._h:
            raise RuntimeError("oracle: " + lib().orc_last_error().decode())
        self.model_dir = model_dir
        g = lambda k: lib().orc_config_int(self._h, k.encode())
        self.D = g("hidden_size")
        self.V = g("vocab_size")
        self.L = g("num_hidden_layers")
        self.E = g("num_experts")
        self.K = g("num_experts_per_tok")
        self.interval = g("full_attention_interval")
        self.nv = g("linear_num_value_heads")
        self.dv = g("linear_value_head_dim")
        self.dk = g("linear_key_head_dim")
        self.cfg = g

    def __del__(self):
        if getattr(self, "_h", None):
            lib().orc_close(self._h)
            self._h = None

    def is_linear_layer(self, i: int) -> bool:
        return (i + 1) % self.interval != 0

    def forward(self, tokens, capture_layers: bool = True) -> dict:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        n = len(t)
        logits = np.zeros((n, self.V), np.float32)
        layers = np.zeros((self.L, n, self.D), np.float32) if capture_layers else None
        emb = np.zeros((n, self.D), np.float32)
        fin = np.zeros((n, self.D), np.float32)
        greedy = np.zeros(n, np.int32)
        picks = np.zeros((self.L, n, self.K), np.int32)
        _check(lib().orc_forward(self._h, _i(t), n, _f(logits), _f(layers) if layers is not None else None,
                                 _f(emb), _f(fin), _i(greedy), _i(picks)))
        return {"logits": logits, "layers": layers, "embed": emb, "final_norm": fin, "greedy": greedy.tolist(),
                "picks": picks}

    def layer_forward(self, h, layer: int, state: DecodeState | None = None) -> np.ndarray:
        h = np.ascontiguousarray(h, dtype=np.float32).reshape(-1, self.D)
        out = np.zeros_like(h)
        _check(lib().orc_layer_forward(self._h, _f(h), h.shape[0], layer, state._h if state else None, _f(out)))
        return out

    def moe_forward(self, x, layer: int):
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, self.D)
        S = x.shape[0]
        out = np.zeros_like(x)
        ids = np.zeros((S, self.K), np.int32)
        pp = np.zeros((S, self.K), np.float32)
        probs = np.zeros((S, self.E), np.float32)
        _check(lib().orc_moe_forward(self._h, layer, _f(x), S, _f(out), _i(ids), _f(pp), _f(probs)))
        return out, ids, pp, probs

    def mixer_forward(self, x, layer: int, state: DecodeState | None = None) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, self.D)
        out = np.zeros_like(x)
        _check(lib().orc_mixer_forward(self._h, layer, _f(x), x.shape[0], state._h if state else None, _f(out)))
        return out

    def delta_state(self, state: DecodeState, layer: int) -> np.ndarray:
        out = np.zeros((self.nv, self.dv, self.dk), np.float32)
        lib().orc_state_delta(self._h, state._h, layer, _f(out))
        return out

    def step(self, tokens, state: DecodeState) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        logits = np.zeros(self.V, np.float32)
        _check(lib().orc_step(self._h, state._h, _i(t), len(t), _f(logits)))
        return logits

    def route_gap(self, reset: bool = False) -> float:
        """Smallest relative gap (p_k - p_k+1) / p_k between the k-th and
        (k+1)-th router probability of any row routed since the last reset:
        below the float noise of the router logits, another implementation's
        top-k may legitimately pick the other expert."""
        return float(lib().orc_route_gap(self._h, int(reset)))

    def tensor_info(self, name: str):
        dt = C.create_string_buffer(8)
        shape = (C.c_int64 * 8)()
        nd = lib().orc_tensor_info(self._h, name.encode(), dt, shape)
        if nd < 0:
            raise RuntimeError("oracle: " + lib().orc_last_error().decode())
        return dt.value.decode(), [shape[i] for i in range(nd)]

    def tensor_bytes(self, name: str, e0: int, e1: int) -> bytes:
        dt, _ = self.tensor_info(name)
        eb = {"F32": 4, "U32": 4, "I32": 4, "BF16": 2, "F16": 2}[dt]
        buf = C.create_string_buffer((e1 - e0) * eb)
        _check(lib().orc_tensor_bytes(self._h, name.encode(), e0, e1, buf))
        return buf.raw

    def dequant(self, path: str, r0: int, r1: int, cols: int) -> np.ndarray:
        out = np.zeros((r1 - r0, cols), np.float32)
        _check(lib().orc_dequant(self._h, path.encode(), r0, r1, _f(out)))
        return out


def gemv_affine(packed, scales, biases, out_dim, in_dim, group, bits, x):
    """Model-free affine GEMV oracle (MetalKernelTests.swift:136-151)."""
    packed = np.ascontiguousarray(packed, dtype=np.uint32)
    sd = {np.dtype(np.float32): 0, np.dtype(np.uint16): 1, np.dtype(np.float16): 2}[scales.dtype]
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(out_dim, np.float32)
    lib().orc_gemv_affine(packed.ctypes.data_as(C.POINTER(C.c_uint32)), scales.ctypes.data, biases.ctypes.data, sd,
                          out_dim, in_dim, group, bits, _f(x), _f(y))
    return y


def expert_swiglu(gate, up, down, D, I, group, bits, x):
    """y = down(silu(gate x) * up x) for one MLX-affine expert; each matrix is (packed, scales, biases)."""
    arrs = [np.ascontiguousarray(a) for m in (gate, up, down) for a in m]
    sd = {np.dtype(np.float32): 0, np.dtype(np.uint16): 1, np.dtype(np.float16): 2}[arrs[1].dtype]
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(D, np.float32)
    lib().orc_expert_swiglu(*[a.ctypes.data for a in arrs], sd, bits, group, D, I, _f(x), _f(y))
    return y


def gated_delta(q, k, v, g, beta, state, T, Hk, Hv, Dk, Dv):
    """Gated delta rule over T steps (gated_delta.py ops path). Returns (y, state)."""
    arrs = [np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v, g, beta)]
    st = np.array(state, dtype=np.float32, copy=True)
    y = np.zeros(T * Hv * Dv, np.float32)
    lib().orc_gated_delta(*[_f(a) for a in arrs], _f(st), _f(y), T, Hk, Hv, Dk, Dv)
    return y, st
