"""The router entry point without a workspace (lmoe_fused_gate_topk_static) against the
workspace entry point, through the C ABI.  This file is collected last on purpose: it must
pass both alone in a fresh process and after every other GPU test has run."""
import numpy as np
import pytest
import torch

from light_moe_b200 import capi

pytestmark = pytest.mark.gpu

STATIC_MAX_TOKENS = 16384


def _outputs(T, E, k, dev):
    return dict(
        ids=torch.full((T, k), -1, dtype=torch.int32, device=dev),
        weights=torch.full((T, k), -1.0, dtype=torch.float32, device=dev),
        weights_bf16=torch.zeros(T, k, dtype=torch.bfloat16, device=dev),
        counts=torch.full((E,), -1, dtype=torch.int32, device=dev),
        offsets=torch.full((E + 1,), -1, dtype=torch.int32, device=dev),
        sorted_idx=torch.full((T * k,), -1, dtype=torch.int32, device=dev),
        positions=torch.full((T * k,), -1, dtype=torch.int32, device=dev),
        logits=torch.zeros(T, E, dtype=torch.float32, device=dev),
    )


def _args(o):
    names = ("ids", "weights", "weights_bf16", "counts", "offsets", "sorted_idx", "positions", "logits")
    return tuple(capi.ptr(o.get(n)) for n in names)


def _select(o, perm, logits):
    # leave out the permutation outputs (non-cooperative launch) and / or the logits (the
    # small-batch path then keeps its fp32 logits in the scratch itself)
    drop = (() if perm else ("counts", "offsets", "sorted_idx", "positions")) + (() if logits else ("logits",))
    return {n: t for n, t in o.items() if n not in drop}


def _route_static(x, w, bias, k, perm=True, logits=True):
    T, d = x.shape
    E = w.shape[0]
    o = _select(_outputs(T, E, k, x.device), perm, logits)
    capi.call("lmoe_fused_gate_topk_static", x.data_ptr(), w.data_ptr(), capi.ptr(bias), T, d, E, k, *_args(o),
              capi.stream_handle())
    torch.cuda.synchronize()
    return {n: t.float().cpu().numpy() if t.dtype == torch.bfloat16 else t.cpu().numpy() for n, t in o.items()}


def _route_workspace(x, w, bias, k, perm=True, logits=True):
    T, d = x.shape
    E = w.shape[0]
    o = _select(_outputs(T, E, k, x.device), perm, logits)
    nbytes = capi.lib().lmoe_router_workspace_bytes(T, E)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=x.device)
    capi.call("lmoe_fused_gate_topk", x.data_ptr(), w.data_ptr(), capi.ptr(bias), T, d, E, k, *_args(o),
              ws.data_ptr(), ws.numel(), capi.stream_handle())
    torch.cuda.synchronize()
    err = np.zeros(1, np.uint32)
    capi.call("lmoe_read_error", ws.data_ptr(), err.ctypes.data, capi.stream_handle())
    assert err[0] == 0, hex(int(err[0]))
    return {n: t.float().cpu().numpy() if t.dtype == torch.bfloat16 else t.cpu().numpy() for n, t in o.items()}


def test_static_router_matches_workspace_router_on_consecutive_calls():
    torch.manual_seed(11)
    dev = torch.device("cuda")
    # the second call is smaller and has fewer experts, so it runs on whatever the first
    # call left in the shared scratch
    # (T, d, E, k, bias, permutation outputs, logits output); T <= 128 runs the small-batch
    # kernels, whose fp32 logits live in the scratch when the caller passes no logits buffer
    cases = [(STATIC_MAX_TOKENS, 1024, 64, 6, True, True, True), (333, 4096, 8, 2, False, True, True),
             (64, 4096, 8, 2, False, True, False), (64, 512, 16, 4, True, False, False),
             (5000, 1024, 8, 2, True, False, True)]
    for T, d, E, k, with_bias, perm, logits in cases:
        x = (torch.randn(T, d, device=dev) * 0.5).to(torch.bfloat16)
        w = (torch.randn(E, d, device=dev) * 0.02).to(torch.bfloat16)
        bias = torch.randn(E, device=dev) * 0.1 if with_bias else None
        a = _route_static(x, w, bias, k, perm, logits)
        b = _route_workspace(x, w, bias, k, perm, logits)
        assert set(a) == set(b)
        # same kernel on the same inputs: the integer outputs are identical and the floating
        # ones agree to the bit (tolerance 0)
        for name in ("ids", "counts", "offsets", "sorted_idx", "positions"):
            if name in a:
                np.testing.assert_array_equal(a[name], b[name], err_msg=f"{name} T={T} E={E}")
        for name in ("weights", "weights_bf16", "logits"):
            if name in a:
                np.testing.assert_allclose(a[name], b[name], rtol=0, atol=0, err_msg=f"{name} T={T} E={E}")
        if perm:
            assert int(a["offsets"][-1]) == T * k


def test_static_router_rejects_more_tokens_than_its_scratch_holds():
    lib = capi.lib()
    st = lib.lmoe_fused_gate_topk_static(None, None, None, STATIC_MAX_TOKENS + 1, 4096, 8, 2, None, None, None,
                                         None, None, None, None, None, None)
    assert st == capi.LMOE_ERR_WORKSPACE
    assert b"workspace" in lib.lmoe_status_string(st)
