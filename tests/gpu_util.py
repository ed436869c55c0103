"""Helpers for the GPU tests: calls through the C ABI (ctypes) on torch-allocated buffers."""
from __future__ import annotations

import numpy as np
import torch

from light_moe_b200 import capi


def stream():
    return capi.stream_handle()


def read_error(ws: torch.Tensor) -> int:
    out = np.zeros(1, np.uint32)
    capi.call("lmoe_read_error", ws.data_ptr(), out.ctypes.data, stream())
    return int(out[0])


def router(x, w, k, bias=None, perm=True, logits=True, positions=False, probs=False):
    """lmoe_fused_gate_topk_typed through the C ABI (x and w of any of bf16 / fp16 / fp32);
    returns numpy arrays."""
    T, d = x.shape
    E = w.shape[0]
    dev = x.device
    xdt, wdt = capi.dtype_code(x.dtype), capi.dtype_code(w.dtype)
    ids = torch.empty(T, k, dtype=torch.int32, device=dev)
    wts = torch.empty(T, k, dtype=torch.float32, device=dev)
    wbf = torch.empty(T, k, dtype=torch.bfloat16, device=dev)
    counts = torch.empty(E, dtype=torch.int32, device=dev) if perm else None
    offsets = torch.empty(E + 1, dtype=torch.int32, device=dev) if perm else None
    sidx = torch.empty(max(T * k, 1), dtype=torch.int32, device=dev) if perm else None
    lg = torch.empty(T, E, dtype=torch.float32, device=dev) if logits else None
    pos = torch.empty(max(T * k, 1), dtype=torch.int32, device=dev) if positions else None
    pr = torch.empty(T, E, dtype=torch.float32, device=dev) if probs else None
    nbytes = capi.lib().lmoe_router_workspace_bytes_typed(T, E, xdt, wdt)
    ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=dev)
    capi.call("lmoe_fused_gate_topk_typed", x.data_ptr(), xdt, w.data_ptr(), wdt, capi.ptr(bias), T, d, E, k,
              ids.data_ptr(),
              wts.data_ptr(), wbf.data_ptr(), capi.ptr(counts), capi.ptr(offsets), capi.ptr(sidx), capi.ptr(pos),
              capi.ptr(lg), capi.ptr(pr),
              ws.data_ptr(), ws.numel(), stream())
    torch.cuda.synchronize()
    err = read_error(ws)
    assert err == 0, hex(err)
    out = dict(ids=ids.cpu().numpy(), weights=wts.cpu().numpy(), weights_bf16=wbf.float().cpu().numpy())
    if perm:
        out.update(counts=counts.cpu().numpy(), offsets=offsets.cpu().numpy(), sorted_idx=sidx[: T * k].cpu().numpy())
    if logits:
        out["logits"] = lg.cpu().numpy()
    if positions:
        out["positions"] = pos[: T * k].cpu().numpy()
    if probs:
        out["probs"] = pr.cpu().numpy()
    return out


def quantize(w, group_size):
    rows = w.numel() // w.shape[-1]
    K = w.shape[-1]
    q = torch.empty(*w.shape[:-1], K // 2, dtype=torch.uint8, device=w.device)
    s = torch.empty(*w.shape[:-1], K // group_size, dtype=torch.float16, device=w.device)
    capi.call("lmoe_quantize_w4", w.data_ptr(), 1 if w.dtype == torch.float32 else 0, rows, K, group_size,
              q.data_ptr(), s.data_ptr(), stream())
    return q, s


def dequantize(q, s, group_size):
    K = q.shape[-1] * 2
    rows = q.numel() // (K // 2)
    out = torch.empty(*q.shape[:-1], K, dtype=torch.bfloat16, device=q.device)
    capi.call("lmoe_dequantize_w4", q.data_ptr(), s.data_ptr(), rows, K, group_size, out.data_ptr(), stream())
    return out


def prepack(q, s, group_size, q_up=None, s_up=None):
    import ctypes
    E, N, K2 = q.shape
    K = K2 * 2
    pb = ctypes.c_size_t()
    capi.call("lmoe_w4_prepacked_bytes", E, N, K, group_size, 1 if q_up is not None else 0, ctypes.byref(pb))
    packed = torch.empty(pb.value, dtype=torch.uint8, device=q.device)
    capi.call("lmoe_prepack_w4", q.data_ptr(), s.data_ptr(), capi.ptr(q_up), capi.ptr(s_up), E, N, K, group_size,
              packed.data_ptr(), stream())
    return packed


def w4_gemm(x, packed, N, group_size, offsets, epilogue=0, dest=None, row_scale=None, out_rows=None,
            hint=0, seg_expert=None, pad=0):
    """``pad`` extra output columns make the row stride ldo = ncols + pad (the returned view
    drops them; they must stay zero)."""
    import ctypes
    R, K = x.shape
    E = offsets.numel() - 1
    ncols = N // 2 if epilogue == 1 else N
    rows_out = out_rows if out_rows is not None else R
    full = torch.zeros(rows_out, ncols + pad, dtype=torch.bfloat16, device=x.device)
    ws = torch.zeros(256, dtype=torch.uint8, device=x.device)
    per = ctypes.c_size_t()
    capi.call("lmoe_w4_prepacked_bytes", 1, N, K, group_size, 0, ctypes.byref(per))
    num_w = packed.numel() // per.value
    capi.call("lmoe_w4a16_grouped_gemm", x.data_ptr(), R, K, packed.data_ptr(), N, group_size,
              offsets.data_ptr(), 1 if offsets.dtype == torch.int64 else 0, E, capi.ptr(seg_expert), num_w,
              epilogue,
              capi.ptr(dest),
              capi.ptr(row_scale), hint, full.data_ptr(), ncols + pad, ws.data_ptr(), ws.numel(), stream())
    torch.cuda.synchronize()
    assert read_error(ws) == 0
    if pad:
        assert torch.all(full[:, ncols:] == 0), "wrote past the output columns"
    return full[:, :ncols]


def bf16_gemm(x, w, offsets, zero_fill=1):
    R, K = x.shape
    E, N, _ = w.shape
    out = torch.empty(R, N, dtype=torch.bfloat16, device=x.device)
    ws = torch.zeros(256, dtype=torch.uint8, device=x.device)
    capi.call("lmoe_grouped_gemm_bf16", x.data_ptr(), R, K, w.data_ptr(), N, offsets.data_ptr(),
              1 if offsets.dtype == torch.int64 else 0, E, zero_fill, out.data_ptr(), ws.data_ptr(), ws.numel(),
              stream())
    torch.cuda.synchronize()
    assert read_error(ws) == 0
    return out


def dense_gemm(x, w, offsets, zero_fill=1):
    """lmoe_grouped_gemm in the dtype of x (bf16 / fp16 / fp32)."""
    R, K = x.shape
    E, N, _ = w.shape
    out = torch.empty(R, N, dtype=x.dtype, device=x.device)
    ws = torch.zeros(256, dtype=torch.uint8, device=x.device)
    capi.call("lmoe_grouped_gemm", x.data_ptr(), capi.dtype_code(x.dtype), R, K, w.data_ptr(), N,
              offsets.data_ptr(), 1 if offsets.dtype == torch.int64 else 0, E, zero_fill, out.data_ptr(),
              ws.data_ptr(), ws.numel(), stream())
    torch.cuda.synchronize()
    assert read_error(ws) == 0
    return out


def layer(x, gate_w, experts, top_k, gate_bias=None):
    """lmoe_moe_layer_w4a16 through the C ABI; returns (y, ids, weights) torch tensors."""
    T, d = x.shape
    E = gate_w.shape[0]
    e = experts
    y = torch.empty(T, d, dtype=torch.bfloat16, device=x.device)
    ids = torch.empty(T, top_k, dtype=torch.int32, device=x.device)
    wts = torch.empty(T, top_k, dtype=torch.float32, device=x.device)
    nbytes = capi.lib().lmoe_moe_layer_workspace_bytes(T, d, e.ffn_size, E, top_k, e.num_shared)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    capi.call("lmoe_moe_layer_w4a16", x.data_ptr(), T, d, gate_w.data_ptr(), capi.ptr(gate_bias), E, top_k,
              e.num_shared, e.w13_packed.data_ptr(), e.w2_packed.data_ptr(), e.ffn_size, e.group_size, y.data_ptr(), ids.data_ptr(), wts.data_ptr(),
              ws.data_ptr(), ws.numel(), stream())
    torch.cuda.synchronize()
    assert read_error(ws) == 0
    return y, ids, wts


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
