"""ctypes binding of the CPU oracle (oracle/oracle.cpp).

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and
``bench.py`` (cpu_baseline and the ``--impl reference`` arm) as the checker /
CPU baseline. The product path never imports this module.

The oracle restates the reference's CPU code (src/quant.rs, src/qwen35.rs,
src/qwen35_runtime.rs, src/metal.rs CPU test restatements, src/runtime.rs
argmax); see the file:line citations in oracle.cpp.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

GGML_F32, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K = 0, 12, 13, 14
BLOCK_BYTES = {GGML_Q4_K: 144, GGML_Q5_K: 176, GGML_Q6_K: 210}

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")


def build(force: bool = False) -> str:
    src = os.path.join(_HERE, "oracle.cpp")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", _HERE, "liboracle.so"])
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        sz, i32, u32 = C.c_size_t, C.c_int, C.c_uint32
        L.or_dequantize.argtypes = [u32, C.c_void_p, sz, sz, _f32p]
        L.or_matvec.argtypes = [u32, C.c_void_p, sz, sz, _f32p, _f32p, i32]
        L.or_fused_gate_up.argtypes = [C.c_void_p, C.c_void_p, sz, sz, _f32p, _f32p, i32]
        L.or_fused_mlp.argtypes = [u32, C.c_void_p, C.c_void_p, u32, C.c_void_p, sz, sz, _f32p, _f32p, i32]
        L.or_rms_norm_heads.argtypes = [_f32p, _f32p, sz, sz, C.c_float, _f32p]
        L.or_gated_rms_norm.argtypes = [_f32p, _f32p, _f32p, sz, sz, C.c_float, _f32p]
        L.or_causal_conv1d_step.argtypes = [_f32p, _f32p, _f32p, sz, sz, _f32p]
        L.or_gdn_step.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, sz, sz, sz, _f32p]
        L.or_rope.argtypes = [_f32p, sz, sz, sz, C.c_float, _f32p]
        L.or_attention_decode.argtypes = [_f32p, C.c_void_p, C.c_void_p, i32, _f32p, _f32p,
                                          sz, sz, sz, sz, sz, _f32p]
        L.or_argmax.argtypes = [_f32p, sz]
        L.or_argmax.restype = C.c_long
        L.or_f32_to_bf16.argtypes = [C.c_float]
        L.or_f32_to_bf16.restype = C.c_uint16
        L.or_model_create.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, i32]
        L.or_model_create.restype = C.c_void_p
        L.or_model_destroy.argtypes = [C.c_void_p]
        L.or_model_embed.argtypes = [C.c_void_p, u32, _f32p]
        L.or_model_decode_hidden.argtypes = [C.c_void_p, sz, _f32p]
        L.or_model_logits.argtypes = [C.c_void_p, _f32p, _f32p]
        L.or_model_generate.argtypes = [C.c_void_p, C.c_void_p, sz, sz, C.c_void_p]
        L.or_model_generate.restype = C.c_long
        L.or_gdn_layer.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, _f32p, _f32p, _f32p,
                                   C.c_void_p, _f32p, i32]
        L.or_attention_layer.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, _f32p, sz,
                                         C.c_void_p, C.c_void_p, C.POINTER(sz), _f32p, i32]
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(C.c_void_p) if isinstance(a, np.ndarray) else a


class OracleError(RuntimeError):
    pass


def _check(rc, what):
    if rc != 0:
        raise OracleError(f"{what} failed with status {rc}")


def dequantize(ggml_type: int, data: np.ndarray, elements: int) -> np.ndarray:
    data = np.ascontiguousarray(data, dtype=np.uint8)
    out = np.empty(max(elements, 1), np.float32)
    _check(lib().or_dequantize(ggml_type, _ptr(data), data.size, elements, out), "dequantize")
    return out[:elements]


def matvec(ggml_type: int, w, rows: int, cols: int, x: np.ndarray, threads: int = 0) -> np.ndarray:
    y = np.empty(rows, np.float32)
    _check(lib().or_matvec(ggml_type, _ptr(w), rows, cols, np.ascontiguousarray(x, np.float32), y, threads), "matvec")
    return y


def matmul_many(ggml_type: int, w, rows: int, cols: int, batch: int, inputs, threads: int = 0) -> np.ndarray:
    """si_q{4,5,6}_k_matmul_many (metal.rs:1083-1127): candidate k's output is
    the dequantised matrix times inputs[k]; one oracle matvec per candidate.
    Returns batch x rows."""
    x = np.ascontiguousarray(inputs, np.float32).reshape(batch, cols)
    return np.stack([matvec(ggml_type, w, rows, cols, x[k], threads) for k in range(batch)])


def fused_gate_up(gate, up, rows, cols, x, threads=0):
    out = np.empty(rows, np.float32)
    _check(lib().or_fused_gate_up(_ptr(gate), _ptr(up), rows, cols, np.ascontiguousarray(x, np.float32), out, threads), "gate_up")
    return out


def fused_mlp(gate_type, gate, up, down_type, down, inter, hidden, x, threads=0):
    y = np.empty(hidden, np.float32)
    _check(lib().or_fused_mlp(gate_type, _ptr(gate), _ptr(up), down_type, _ptr(down), inter, hidden,
                              np.ascontiguousarray(x, np.float32), y, threads), "mlp")
    return y


def rms_norm_heads(x, w, heads, hd, eps):
    out = np.empty(heads * hd, np.float32)
    _check(lib().or_rms_norm_heads(np.ascontiguousarray(x, np.float32), np.ascontiguousarray(w, np.float32), heads, hd, eps, out), "rms_norm_heads")
    return out


def gated_rms_norm(x, g, w, heads, hd, eps):
    out = np.empty(heads * hd, np.float32)
    _check(lib().or_gated_rms_norm(np.ascontiguousarray(x, np.float32), np.ascontiguousarray(g, np.float32),
                                   np.ascontiguousarray(w, np.float32), heads, hd, eps, out), "gated_rms_norm")
    return out


def causal_conv1d_step(x, state, w, channels, kernel):
    """Returns (out, new_state); `state` is not modified."""
    st = np.array(state, np.float32, copy=True)
    out = np.empty(channels, np.float32)
    _check(lib().or_causal_conv1d_step(np.ascontiguousarray(x, np.float32), st, np.ascontiguousarray(w, np.float32),
                                       channels, kernel, out), "conv")
    return out, st


def gdn_step(q, k, v, g, beta, state, heads, kd, vd):
    """Returns (out, new_state); `state` is not modified."""
    st = np.array(state, np.float32, copy=True)
    out = np.empty(heads * vd, np.float32)
    f = lambda a: np.ascontiguousarray(a, np.float32)
    _check(lib().or_gdn_step(st, f(q), f(k), f(v), f(g), f(beta), heads, kd, vd, out), "gdn_step")
    return out, st


def gdn_step_parallel(q, k, v, g, beta, state, heads, kd, vd):
    """si_gated_delta_step_parallel (src/metal.rs:688-740), the reference's
    other formulation of the recurrence: one lane per (head, value column)
    decays its state column while summing memory = S^T k and S^T q over the
    keys in order, then delta = (v - memory) * beta, S += k delta, and
    out = S_decayed^T q + delta * (k . q). f32 throughout; returns (out,
    new_state) without modifying `state`."""
    f32 = np.float32
    q = np.asarray(q, f32).reshape(heads, kd)
    k = np.asarray(k, f32).reshape(heads, kd)
    v = np.asarray(v, f32).reshape(heads, vd)
    st = np.array(state, f32, copy=True).reshape(heads, kd, vd)
    out = np.empty((heads, vd), f32)
    for h in range(heads):
        kq = f32(0)
        for i in range(kd):
            kq = f32(kq + k[h, i] * q[h, i])
        decay = f32(np.exp(f32(g[h])))
        memory = np.zeros(vd, f32)
        qsum = np.zeros(vd, f32)
        for i in range(kd):
            st[h, i] = st[h, i] * decay
            memory = memory + st[h, i] * k[h, i]
            qsum = qsum + st[h, i] * q[h, i]
        delta = (v[h] - memory) * f32(beta[h])
        for i in range(kd):
            st[h, i] = st[h, i] + k[h, i] * delta
        out[h] = qsum + delta * kq
    return out.reshape(-1), st.reshape(-1)


def rope(x, heads, hd, pos, theta):
    out = np.empty(heads * hd, np.float32)
    _check(lib().or_rope(np.ascontiguousarray(x, np.float32), heads, hd, pos, theta, out), "rope")
    return out


def attention_decode(q, kc, vc, nk, nv, qh, kvh, hd, cached, cap):
    """kc/vc: float32 (reference layout) or uint16 (bf16 bits) arrays [kvh][cap][hd]."""
    kc = np.ascontiguousarray(kc)
    vc = np.ascontiguousarray(vc)
    ct = 1 if kc.dtype == np.uint16 else 0
    out = np.empty(qh * hd, np.float32)
    f = lambda a: np.ascontiguousarray(a, np.float32)
    _check(lib().or_attention_decode(f(q), _ptr(kc), _ptr(vc), ct, f(nk), f(nv), qh, kvh, hd, cached, cap, out), "attention")
    return out


def argmax(v) -> int:
    return int(lib().or_argmax(np.ascontiguousarray(v, np.float32), len(v)))


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bits (vectorised restatement)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return r


class OracleModel:
    """The oracle's 64-layer (or smaller) decoder over the host tensors of a
    backend `Model` (its pinned host copy, rank 0 of 1)."""

    def __init__(self, config, host_tensor, threads: int = 0):
        """config: a ctypes si_model_config; host_tensor(layer, id) -> (addr, bytes, type)."""
        L = lib()
        n = (config.layers + 1) * 23
        ptrs = (C.c_void_p * n)()
        types = (C.c_uint32 * n)()
        for layer in range(config.layers + 1):
            for tid in range(23):
                addr, _, ty = host_tensor(layer, tid)
                ptrs[layer * 23 + tid] = addr
                types[layer * 23 + tid] = ty
        self._cfg = config
        self.h = L.or_model_create(C.byref(config), ptrs, types, threads)

    def close(self):
        if self.h:
            lib().or_model_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def embed(self, token):
        out = np.empty(self._cfg.hidden, np.float32)
        _check(lib().or_model_embed(self.h, token, out), "embed")
        return out

    def decode_hidden(self, position, hidden):
        h = np.array(hidden, np.float32, copy=True)
        _check(lib().or_model_decode_hidden(self.h, position, h), "decode_hidden")
        return h

    def logits(self, hidden):
        out = np.empty(self._cfg.vocab, np.float32)
        _check(lib().or_model_logits(self.h, np.ascontiguousarray(hidden, np.float32), out), "logits")
        return out

    def generate(self, prompt, max_new):
        p = np.ascontiguousarray(prompt, np.uint32)
        out = np.zeros(max(max_new, 1), np.uint32)
        n = lib().or_model_generate(self.h, p.ctypes.data_as(C.c_void_p), p.size, max_new,
                                    out.ctypes.data_as(C.c_void_p))
        if n < 0:
            raise OracleError(f"generate failed with {n}")
        return out[:n].tolist()


def _tensor_table(tensors):
    """tensors: {tensor id: (numpy array, ggml type)} -> ctypes pointer/type arrays (23 ids)."""
    ptrs = (C.c_void_p * 23)()
    types = (C.c_uint32 * 23)()
    for tid, (arr, ty) in tensors.items():
        ptrs[tid] = arr.ctypes.data
        types[tid] = ty
    return ptrs, types


def gdn_layer(config, tensors, x, conv_state, rec_state, gates=None, threads: int = 0):
    """gdn_token_mixer (qwen35_runtime.rs:409-624) on one token: x is the mixer
    input; conv_state ([channels][kernel-1]) and rec_state ([vh][128][128]) are
    updated in place; gates, if given, is [g[vh], beta[vh]] used as is.
    Returns the mixer output [hidden]."""
    ptrs, types = _tensor_table(tensors)
    out = np.empty(config.hidden, np.float32)
    g = None if gates is None else np.ascontiguousarray(gates, np.float32)
    _check(lib().or_gdn_layer(C.byref(config), ptrs, types, np.ascontiguousarray(x, np.float32), conv_state,
                              rec_state, None if g is None else g.ctypes.data_as(C.c_void_p), out, threads),
           "gdn_layer")
    return out


def attention_layer(config, tensors, x, position, kc, vc, cached, threads: int = 0):
    """attention_token_mixer (qwen35_runtime.rs:628-867) over bf16 head-major
    caches kc/vc ([kvh][kv_capacity][hd], uint16, appended in place at
    `cached`). Returns (mixer output [hidden], new cached count)."""
    ptrs, types = _tensor_table(tensors)
    out = np.empty(config.hidden, np.float32)
    n = C.c_size_t(cached)
    _check(lib().or_attention_layer(C.byref(config), ptrs, types, np.ascontiguousarray(x, np.float32), position,
                                    kc.ctypes.data_as(C.c_void_p), vc.ctypes.data_as(C.c_void_p), C.byref(n), out,
                                    threads), "attention_layer")
    return out, n.value
