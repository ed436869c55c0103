"""CPU tests of the C ABI boundary: the library loads, exports every function that
include/lmoe_b200.h declares, the ctypes signature table covers them, the host-only entry
points compute sizes, and argument validation rejects bad calls before touching a GPU."""
import ctypes
import os
import re

import pytest

from light_moe_b200 import capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "lmoe_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lmoe_\w+)\s*\(", text)))


def test_library_exports_every_declared_function():
    lib = capi.lib()
    names = declared_functions()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), f"{n} declared in the header but not exported"


def test_signature_table_matches_header():
    assert set(capi.SIGNATURES) == set(declared_functions())


def test_extension_module_exposes_reference_ops():
    from light_moe_b200 import ops
    ext = ops.extension()
    for name in ("grouped_gemm", "fused_gate_topk", "fused_gate_topk_permute", "fused_gate_topk_ex",
                 "quantize_w4", "dequantize_w4", "prepack_w4", "w4a16_grouped_gemm", "combine_rows",
                 "moe_layer_w4a16"):
        assert hasattr(ext, name)
    doc = ext.fused_gate_topk.__doc__
    assert "hidden_states" in doc and "gate_weight" in doc and "top_k" in doc


def test_host_only_entry_points():
    lib = capi.lib()
    assert lib.lmoe_version() >= 100
    assert lib.lmoe_status_string(0) == b"ok"
    assert b"workspace" in lib.lmoe_status_string(capi.LMOE_ERR_WORKSPACE)
    # router scratch: 256 B header + per-tile counts + per-tile bitmaps, for at most
    # max(ceil(T/128), min(ceil(T/8), 256)) tiles (tiles shrink below 128 tokens to fill the SMs)
    assert lib.lmoe_router_workspace_bytes(16384, 64) == 256 + 256 * 64 * 4 + 256 * 64 * 16
    assert lib.lmoe_router_workspace_bytes(65536, 8) == 256 + 512 * 8 * 4 + 512 * 8 * 16
    assert lib.lmoe_router_workspace_bytes(1000, 8) == (256 + 125 * 8 * 4 + 255) // 256 * 256 + 125 * 8 * 16
    assert lib.lmoe_router_workspace_bytes(-1, 8) == 0
    nb = ctypes.c_size_t()
    # Mixtral gate/up: 8 experts, 2 x 14336 rows x 4096 K, g=128: 8192 B int4 + 256 B scales per super-block
    assert lib.lmoe_w4_prepacked_bytes(8, 14336, 4096, 128, 1, ctypes.byref(nb)) == 0
    assert nb.value == 8 * (2 * 14336 // 128) * (4096 // 128) * (8192 + 256)
    assert nb.value == 8 * 2 * 14336 * 4096 // 2 + 8 * 2 * 14336 * (4096 // 128) * 2  # == canonical bytes
    # g = 64: two scale groups per super-block
    assert lib.lmoe_w4_prepacked_bytes(2, 128, 256, 64, 0, ctypes.byref(nb)) == 0
    assert nb.value == 2 * 1 * 2 * (8192 + 512)
    # unsupported layouts are rejected
    assert lib.lmoe_w4_prepacked_bytes(2, 100, 256, 64, 0, ctypes.byref(nb)) == capi.LMOE_ERR_INVALID_ARG
    assert lib.lmoe_w4_prepacked_bytes(2, 128, 192, 64, 0, ctypes.byref(nb)) == capi.LMOE_ERR_INVALID_ARG
    assert lib.lmoe_gemm_workspace_bytes() == 256
    assert lib.lmoe_moe_layer_workspace_bytes(64, 4096, 14336, 8, 2, 0) > 128 * 14336 * 2


@pytest.mark.parametrize("args", [
    # (T, d, E, k): top_k > E, E > 256, d not a multiple of 64, top_k > 16
    (16, 128, 4, 5), (16, 128, 300, 2), (16, 100, 8, 2), (16, 128, 64, 17),
])
def test_router_rejects_bad_arguments_without_gpu(args):
    T, d, E, k = args
    lib = capi.lib()
    st = lib.lmoe_fused_gate_topk(None, None, None, T, d, E, k, None, None, None, None, None, None, None, None,
                                  None, 0, None)
    assert st == capi.LMOE_ERR_INVALID_ARG


def test_layer_rejects_bad_arguments_without_gpu():
    lib = capi.lib()
    # ffn not a multiple of 128
    st = lib.lmoe_moe_layer_w4a16(None, 64, 4096, None, None, 8, 2, 0, None, None, 14300, 128, None, None, None,
                                  None, 0, None)
    assert st == capi.LMOE_ERR_INVALID_ARG
    with pytest.raises(capi.LmoeError):
        capi.call("lmoe_combine_rows", None, None, None, 4, 2, 7, None, 0, None, None)


def test_gemm_sm_limit_is_process_wide_and_validated():
    lib = capi.lib()
    prev = lib.lmoe_get_gemm_sm_limit()
    try:
        assert lib.lmoe_set_gemm_sm_limit(132) == 0 and lib.lmoe_get_gemm_sm_limit() == 132
        assert lib.lmoe_set_gemm_sm_limit(-1) == capi.LMOE_ERR_INVALID_ARG
        assert lib.lmoe_get_gemm_sm_limit() == 132
        assert lib.lmoe_set_gemm_sm_limit(0) == 0 and lib.lmoe_get_gemm_sm_limit() == 0
    finally:
        lib.lmoe_set_gemm_sm_limit(prev)
