"""TEST INFRASTRUCTURE ONLY: numpy/ctypes front end of the C oracle
(attn_oracle.c), the CPU restatement of the lisa-rs attention shaders.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module. The product path (lisa-rs_b200/lisa_attn.py and the CUDA
library) never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libattn_oracle.so")
_lib = None

QH, KVH, HD = 24, 4, 256


def build() -> str:
    """Compile libattn_oracle.so with the Makefile beside this file."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        u32, i32, f32 = ctypes.c_uint32, ctypes.c_int, ctypes.c_float
        L.orc_q_prologue.argtypes = [P, i32, u32, P, f32, P, P]
        L.orc_kv_append.argtypes = [P, P, i32, u32, P, f32, P, P, u32]
        L.orc_sdpa_serial.argtypes = [P, P, P, u32, u32, i32, P]
        L.orc_sdpa_sliced.argtypes = [P, P, P, u32, u32, i32, P]
        L.orc_gate.argtypes = [P, P, i32, P]
        L.orc_attention_layer.argtypes = [P, P, P, i32, u32, P, P, f32, P, P, u32, i32, P]
        L.orc_legacy_batch.argtypes = [P, P, P, i32, P, P, f32, P]
        L.orc_rope_inv_freq.argtypes = [i32]
        L.orc_rope_inv_freq.restype = f32
        L.orc_num_threads.restype = i32
        L.orc_set_num_threads.argtypes = [i32]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


# ---- bf16 helpers (numpy) --------------------------------------------------

def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(f: np.ndarray) -> np.ndarray:
    """Round to nearest even (the device-side bfloat(float) rule)."""
    u = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def f32_to_bf16_trunc(f: np.ndarray) -> np.ndarray:
    """Truncation, as lisa-rs src/format/dtype.rs:42-47 (test fixtures only)."""
    return (np.ascontiguousarray(f, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


# ---- wrappers --------------------------------------------------------------

def q_prologue(q_gate, base, q_norm_w, eps=1e-6):
    q_gate = np.ascontiguousarray(q_gate, dtype=np.float32).reshape(-1, QH * 512)
    rows = q_gate.shape[0]
    query = np.zeros((rows, QH, HD), np.uint16)
    gate = np.zeros((rows, QH, HD), np.float32)
    lib().orc_q_prologue(_p(q_gate), rows, base, _p(np.ascontiguousarray(q_norm_w, np.uint16)),
                         eps, _p(query), _p(gate))
    return query, gate


def kv_append(k, v, base, k_norm_w, k_cache, v_cache, eps=1e-6):
    """Appends in place. k_cache/v_cache uint16 [4][cap][256]."""
    k = np.ascontiguousarray(k, dtype=np.float32).reshape(-1, KVH * HD)
    v = np.ascontiguousarray(v, dtype=np.float32).reshape(-1, KVH * HD)
    cap = k_cache.shape[1]
    lib().orc_kv_append(_p(k), _p(v), k.shape[0], base, _p(np.ascontiguousarray(k_norm_w, np.uint16)),
                        eps, _p(k_cache), _p(v_cache), cap)


def sdpa(query, k_cache, v_cache, base, sliced=True):
    query = np.ascontiguousarray(query, dtype=np.uint16).reshape(-1, QH, HD)
    rows = query.shape[0]
    out = np.zeros((rows, QH, HD), np.float32)
    fn = lib().orc_sdpa_sliced if sliced else lib().orc_sdpa_serial
    fn(_p(query), _p(k_cache), _p(v_cache), k_cache.shape[1], base, rows, _p(out))
    return out


def gate_out(out, gate):
    out = np.ascontiguousarray(out, np.float32)
    gate = np.ascontiguousarray(gate, np.float32)
    gated = np.zeros(out.shape, np.uint16)
    lib().orc_gate(_p(out), _p(gate), out.size, _p(gated))
    return gated


def attention_layer(q_gate, k, v, base, q_norm_w, k_norm_w, k_cache, v_cache, eps=1e-6, sliced=True):
    """Whole layer; appends to the caches in place; returns gated bf16 bits [rows, 6144]."""
    q_gate = np.ascontiguousarray(q_gate, dtype=np.float32).reshape(-1, QH * 512)
    rows = q_gate.shape[0]
    k = np.ascontiguousarray(k, dtype=np.float32).reshape(rows, KVH * HD)
    v = np.ascontiguousarray(v, dtype=np.float32).reshape(rows, KVH * HD)
    gated = np.zeros((rows, QH * HD), np.uint16)
    lib().orc_attention_layer(_p(q_gate), _p(k), _p(v), rows, base,
                              _p(np.ascontiguousarray(q_norm_w, np.uint16)),
                              _p(np.ascontiguousarray(k_norm_w, np.uint16)), eps,
                              _p(k_cache), _p(v_cache), k_cache.shape[1], int(sliced), _p(gated))
    return gated


def legacy_batch(q, k, v, q_norm_w, k_norm_w, eps=1e-6):
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    L = q.shape[0]
    out = np.zeros((L, QH, HD), np.float32)
    lib().orc_legacy_batch(_p(q), _p(k), _p(v), L, _p(np.ascontiguousarray(q_norm_w, np.uint16)),
                           _p(np.ascontiguousarray(k_norm_w, np.uint16)), eps, _p(out))
    return out


def num_threads() -> int:
    return lib().orc_num_threads()


def set_num_threads(n: int) -> None:
    lib().orc_set_num_threads(n)


# ---- affine-u4 QMV (numpy) ---------------------------------------------------

def q4_qmv(x_bits, packed, scale_bits, bias_bits):
    """out[m][n] = sum_k bf16(x[m][k]) * (q[n][k] * scale[n][k/64] + bias[n][k/64]),
    the arithmetic of q4_qmv_fast_impl (src/kernels/shaders/qmv.metal:1-77):
    nibble k%8 of word k/8 (low first), group size 64, bf16 scales / biases.
    Evaluated in float64 (the kernel and the reference sum in f32 in their own
    orders); returns float32 [M, N]."""
    x_bits = np.asarray(x_bits, np.uint16)
    packed = np.asarray(packed, np.uint32)
    m_rows, k = x_bits.shape
    n = packed.shape[0]
    q = ((packed[:, :, None] >> (4 * np.arange(8, dtype=np.uint32))) & 0xF).reshape(n, k).astype(np.float64)
    s = bf16_to_f32(np.asarray(scale_bits, np.uint16).reshape(n, k // 64)).astype(np.float64)
    b = bf16_to_f32(np.asarray(bias_bits, np.uint16).reshape(n, k // 64)).astype(np.float64)
    x = bf16_to_f32(x_bits).astype(np.float64)
    # sum_k x*(q*s+b) = sum_g s_g * sum_{k in g} x q + b_g * sum_{k in g} x
    xq = (x[:, None, :] * q[None, :, :]).reshape(m_rows, n, k // 64, 64).sum(-1)
    xs = x.reshape(m_rows, k // 64, 64).sum(-1)
    out = (xq * s[None]).sum(-1) + (xs[:, None, :] * b[None]).sum(-1)
    return out.astype(np.float32)


# ---- Gated DeltaNet recurrence (numpy) ----------------------------------------

def gdn_recurrence(conv_out, q, k, beta, decay, state, value_heads=48, repeat=3):
    """gdn_recurrence (src/kernels/shaders/gdn.metal:245-330) in float64:
    per token s *= decay; delta = (v - s.k) * beta; s += delta k; y = bf16(s.q).
    state [value_heads, 128, 128] (value col, key dim); returns (y [T, vd]
    float32 bf16-rounded, new state float64)."""
    D = 128
    kd = value_heads // repeat * D
    s = np.asarray(state, np.float64).copy()
    T = conv_out.shape[0]
    y = np.zeros((T, value_heads * D), np.float32)
    for t in range(T):
        kt = k[t].astype(np.float64).reshape(-1, D)[np.arange(value_heads) // repeat]  # [vh, 128]
        qt = q[t].astype(np.float64).reshape(-1, D)[np.arange(value_heads) // repeat]
        v = conv_out[t, 2 * kd:].astype(np.float64).reshape(value_heads, D)
        s *= decay[t].astype(np.float64)[:, None, None]
        kv = np.einsum("hcd,hd->hc", s, kt)
        delta = (v - kv) * beta[t].astype(np.float64)[:, None]
        s += delta[:, :, None] * kt[:, None, :]
        y[t] = bf16_to_f32(f32_to_bf16(np.einsum("hcd,hd->hc", s, qt).reshape(-1).astype(np.float32)))
    return y, s
