"""ctypes bindings of the C oracle (test infrastructure only).

Every function here calls ``lmoe_oracle.c``; see that file for the arithmetic contract and
the light-moe reference lines each step follows.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liblmoe_oracle.so")
_lib = None
_lock = threading.Lock()

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int


def build_oracle(force: bool = False) -> str:
    """Compile the C oracle with its Makefile (gcc); returns the library path."""
    src = os.path.join(_HERE, "lmoe_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def load():
    """Load (building first if needed) the oracle shared library."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                build_oracle()
            lib = ctypes.CDLL(_LIB_PATH)
            lib.lmoe_ref_route.argtypes = [_P, _I32, _I32, _I32, _P, _P]
            lib.lmoe_ref_route.restype = _I32
            lib.lmoe_ref_softmax.argtypes = [_P, _I32, _I32, _P]
            lib.lmoe_ref_softmax.restype = _I32
            lib.lmoe_ref_counts_offsets.argtypes = [_P, _I32, _I32, _I32, _P, _P, _P]
            lib.lmoe_ref_counts_offsets.restype = _I32
            lib.lmoe_ref_quantize_w4.argtypes = [_P, _I64, _I32, _I32, _P, _P]
            lib.lmoe_ref_quantize_w4.restype = _I32
            lib.lmoe_ref_dequantize_w4.argtypes = [_P, _P, _I64, _I32, _I32, _P]
            lib.lmoe_ref_dequantize_w4.restype = _I32
            for name in ("lmoe_ref_f32_to_f16_array", "lmoe_ref_f32_to_bf16_array"):
                getattr(lib, name).argtypes = [_P, _I64, _P]
                getattr(lib, name).restype = None
            lib.lmoe_ref_expf_array.argtypes = [_P, _I64, _P]
            lib.lmoe_ref_expf_array.restype = None
            _lib = lib
    return _lib


def _c(a: np.ndarray, dtype) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=dtype)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def f32_to_bf16_bits(x) -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    load().lmoe_ref_f32_to_bf16_array(_ptr(x), x.size, _ptr(out))
    return out


def bf16_bits_to_f32(b) -> np.ndarray:
    b = _c(b, np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def f32_to_f16_bits(x) -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    load().lmoe_ref_f32_to_f16_array(_ptr(x), x.size, _ptr(out))
    return out


def f16_bits_to_f32(b) -> np.ndarray:
    return _c(b, np.uint16).view(np.float16).astype(np.float32)


def ref_expf(x) -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.float32)
    load().lmoe_ref_expf_array(_ptr(x), x.size, _ptr(out))
    return out


def softmax_probs(logits) -> np.ndarray:
    """The full fp32 softmax probabilities [T, E] with the routing's own arithmetic
    (router_probs of python/light_moe/ops/moe_gate.py:66-67)."""
    lg = _c(logits, np.float32)
    T, E = lg.shape
    out = np.empty((T, E), np.float32)
    if load().lmoe_ref_softmax(_ptr(lg), T, E, _ptr(out)) != 0:
        raise ValueError("oracle softmax: bad arguments")
    return out


def route(logits, top_k: int):
    """Routing from fp32 logits [T, E] -> (ids int32 [T, k], weights fp32 [T, k]).

    Restates csrc/fused_moe_ops.cu:49-134 / python/light_moe/ops/moe_gate.py:39-77 with the
    lower-id tie-break of fused_moe_ops.cu:106-118.
    """
    lg = _c(logits, np.float32)
    T, E = lg.shape
    ids = np.empty((T, top_k), np.int32)
    w = np.empty((T, top_k), np.float32)
    rc = load().lmoe_ref_route(_ptr(lg), T, E, top_k, _ptr(ids), _ptr(w))
    if rc != 0:
        raise ValueError(f"oracle route: bad arguments (E={E}, k={top_k})")
    return ids, w


def counts_offsets(ids, num_experts: int):
    """(counts int32 [E], offsets int32 [E+1], sorted_idx int32 [T*k]) -- stable order.

    Restates python/light_moe/ops/grouped_gemm.py:240-242 (bincount + cumsum) and pins the
    permutation of grouped_gemm.py:233 to (expert, token, slot).
    """
    ids = _c(ids, np.int32)
    T, k = ids.shape
    counts = np.empty(num_experts, np.int32)
    offsets = np.empty(num_experts + 1, np.int32)
    sidx = np.empty(T * k, np.int32)
    rc = load().lmoe_ref_counts_offsets(_ptr(ids), T, k, num_experts, _ptr(counts), _ptr(offsets), _ptr(sidx))
    if rc != 0:
        raise ValueError("oracle counts_offsets: expert id out of range")
    return counts, offsets, sidx


def quantize_w4(w, group_size: int):
    """w [..., N, K] (fp32 values) -> (packed uint8 [..., N, K/2], scales fp16 bits [..., N, K/g])."""
    w = _c(w, np.float32)
    *lead, N, K = w.shape
    rows = int(np.prod(lead, dtype=np.int64)) * N if lead else N
    packed = np.empty((*lead, N, K // 2), np.uint8)
    scales = np.empty((*lead, N, K // group_size), np.uint16)
    rc = load().lmoe_ref_quantize_w4(_ptr(w), rows, K, group_size, _ptr(packed), _ptr(scales))
    if rc != 0:
        raise ValueError("oracle quantize_w4: K must be even and divisible by the group size")
    return packed, scales


def dequantize_w4(packed, scales, group_size: int) -> np.ndarray:
    """-> bf16 bits [..., N, K] with value bf16_rn(q * s)."""
    packed = _c(packed, np.uint8)
    scales = _c(scales, np.uint16)
    *lead, N, K2 = packed.shape
    K = K2 * 2
    rows = int(np.prod(lead, dtype=np.int64)) * N if lead else N
    out = np.empty((*lead, N, K), np.uint16)
    rc = load().lmoe_ref_dequantize_w4(_ptr(packed), _ptr(scales), rows, K, group_size, _ptr(out))
    if rc != 0:
        raise ValueError("oracle dequantize_w4: bad shape")
    return out
