"""ctypes view of the C ABI (include/lmoe_b200.h).

This is the binding a non-PyTorch host (or a test) uses to reach the CUDA library
directly: plain pointers, sizes and a CUDA stream handle.  ``lib()`` loads
``lib/liblmoe_b200.so`` and raises if it is missing -- there is no fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "liblmoe_b200.so")

LMOE_OK = 0
LMOE_ERR_INVALID_ARG = -1
LMOE_ERR_UNSUPPORTED = -2
LMOE_ERR_WORKSPACE = -3
LMOE_ERR_DEVICE = -4

LMOE_DTYPE_BF16 = 0
LMOE_DTYPE_F16 = 1
LMOE_DTYPE_F32 = 2

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/lmoe_b200.h
SIGNATURES = {
    "lmoe_version": (_I, []),
    "lmoe_status_string": (ctypes.c_char_p, [_I]),
    "lmoe_read_error": (_I, [_P, _P, _P]),
    "lmoe_set_gemm_sm_limit": (_I, [_I]),
    "lmoe_capacity_send_plan": (_I, [_P, _P, _P, _I64, _I, _I, _I, _I64, _P, _P, _P]),
    "lmoe_capacity_receive_plan": (_I, [_P, _I, _I, _I64, _I, _I64, _P, _P, _P, _P]),
    "lmoe_p2p_buffer_bytes": (_SZ, [_I, _I, _I64, _I, _I, _I]),
    "lmoe_p2p_buffer_offsets": (_I, [_I, _I, _I64, _I, _I, _I, _P, _P]),
    "lmoe_p2p_alloc": (_I, [_SZ, _P, _P]),
    "lmoe_p2p_open": (_I, [_P, _P]),
    "lmoe_p2p_close": (_I, [_P]),
    "lmoe_p2p_free": (_I, [_P]),
    "lmoe_p2p_exchange_counts": (_I, [_P, _I, _I, _I, _I64, _I, _I, _I, _I64, _P, _P, _P, _P, _P]),
    "lmoe_p2p_dispatch": (_I, [_P, _I, _I, _I, _I64, _I, _I, _I, _I64, _P, _P, _P, _P, _P, _P, _P]),
    "lmoe_p2p_wait": (_I, [_P, _I, _I, _I, _I64, _I, _I, _I, _I64, _P, _I, _P]),
    "lmoe_p2p_send_back": (_I, [_P, _I, _I, _I, _I64, _I, _I, _I, _I64, _P, _P, _P, _P]),
    "lmoe_p2p_init": (_I, [_P, _I, _I, _I, _I64, _I, _I, _I, _P, _P]),
    "lmoe_p2p_down_gemm": (_I, [_P, _I, _I, _I, _I64, _I, _I, _I, _I64, _P, _P, _P, _I, _P, _I, _P, _P, _I,
                                _I, _P, _P]),
    "lmoe_get_gemm_sm_limit": (_I, []),
    "lmoe_router_workspace_bytes": (_SZ, [_I64, _I]),
    "lmoe_router_workspace_bytes_typed": (_SZ, [_I64, _I, _I, _I]),
    "lmoe_fused_gate_topk_typed": (_I, [_P, _I, _P, _I, _P, _I64, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                        _P, _SZ, _P]),
    "lmoe_fused_gate_topk": (_I, [_P, _P, _P, _I64, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "lmoe_fused_gate_topk_static": (_I, [_P, _P, _P, _I64, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "lmoe_permute_rows": (_I, [_P, _I, _P, _I64, _I, _I, _P, _P]),
    "lmoe_quantize_w4": (_I, [_P, _I, _I64, _I, _I, _P, _P, _P]),
    "lmoe_dequantize_w4": (_I, [_P, _P, _I64, _I, _I, _P, _P]),
    "lmoe_w4_prepacked_bytes": (_I, [_I, _I, _I, _I, _I, _P]),
    "lmoe_prepack_w4": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P, _P]),
    "lmoe_gemm_workspace_bytes": (_SZ, []),
    "lmoe_grouped_gemm": (_I, [_P, _I, _I64, _I, _P, _I, _P, _I, _I, _I, _P, _P, _SZ, _P]),
    "lmoe_grouped_gemm_bf16": (_I, [_P, _I64, _I, _P, _I, _P, _I, _I, _I, _P, _P, _SZ, _P]),
    "lmoe_w4a16_grouped_gemm": (_I, [_P, _I64, _I, _P, _I, _I, _P, _I, _I, _P, _I, _I, _P, _P, _I64, _P, _I64, _P,
                                     _SZ, _P]),
    "lmoe_combine_rows": (_I, [_P, _P, _P, _I64, _I, _I, _P, _I, _P, _P]),
    "lmoe_moe_layer_workspace_bytes": (_SZ, [_I64, _I, _I, _I, _I, _I]),
    "lmoe_moe_layer_w4a16": (_I, [_P, _I64, _I, _P, _P, _I, _I, _I, _P, _P, _I, _I, _P, _P, _P, _P, _SZ, _P]),
}

_lib = None
_lock = threading.Lock()


class LmoeError(RuntimeError):
    """A C-ABI call returned a nonzero status."""

    def __init__(self, func: str, status: int):
        msg = lib().lmoe_status_string(status).decode()
        super().__init__(f"{func}: {msg} (status {status})")
        self.status = status


def lib():
    """Load the shared library (raises OSError when it has not been built)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise OSError(f"{LIB_PATH} is missing: build it with `python -m light_moe_b200.build`")
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def call(name: str, *args) -> None:
    """Call an int-returning entry point and raise LmoeError on a nonzero status."""
    st = getattr(lib(), name)(*args)
    if st != LMOE_OK:
        raise LmoeError(name, st)


def ptr(t) -> int | None:
    """Device pointer of a torch tensor (None for None)."""
    return None if t is None else t.data_ptr()


def dtype_code(dtype) -> int:
    """LMOE_DTYPE_* code of a torch floating dtype (bf16, fp16, fp32)."""
    import torch

    codes = {torch.bfloat16: LMOE_DTYPE_BF16, torch.float16: LMOE_DTYPE_F16, torch.float32: LMOE_DTYPE_F32}
    if dtype not in codes:
        raise ValueError(f"unsupported dtype {dtype}")
    return codes[dtype]


def stream_handle(stream=None) -> int:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream
