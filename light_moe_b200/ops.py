"""The light-moe operator surface, backed by the sm_100a library.

Same names, argument names and return types as the reference's ``light_moe._C``
(csrc/bindings.cpp:28-49 of Whitehall945/light-moe):

    grouped_gemm(input, weights, expert_offsets, num_experts) -> Tensor
    fused_gate_topk(hidden_states, gate_weight, top_k) -> (ids int32, weights)
    fused_gate_topk_permute(hidden_states, gate_weight, top_k)
        -> (permuted, ids, weights, offsets int64, sorted_idx int64)

plus the new ops (``fused_gate_topk_ex``, ``quantize_w4``, ``dequantize_w4``, ``prepack_w4``,
``w4a16_grouped_gemm``, ``moe_layer_w4a16``).  Every op runs the CUDA library; if the
``_C`` extension has not been built, calling any op raises -- there is no fallback path.
"""
from __future__ import annotations

import importlib

_ext = None


def extension():
    """The compiled ``_C`` module (raises RuntimeError if it is not built)."""
    global _ext
    if _ext is None:
        try:
            _ext = importlib.import_module("light_moe_b200._C")
        except ImportError as e:  # pragma: no cover - exercised only without a build
            raise RuntimeError(
                "light_moe_b200._C is not built; run `python -m light_moe_b200.build` "
                f"(import error: {e})") from e
    return _ext


def grouped_gemm(input, weights, expert_offsets, num_experts):
    """Dense bf16 grouped GEMM; rows outside every expert range are zero (grouped_gemm.cu:24)."""
    return extension().grouped_gemm(input, weights, expert_offsets, num_experts)


def fused_gate_topk(hidden_states, gate_weight, top_k):
    """(expert_ids int32 [T, k], expert_weights [T, k] in the hidden dtype)."""
    return extension().fused_gate_topk(hidden_states, gate_weight, top_k)


def fused_gate_topk_permute(hidden_states, gate_weight, top_k):
    """(permuted [T*k, d], ids, weights, expert_offsets int64 [E+1], sorted_idx int64 [T*k])."""
    return extension().fused_gate_topk_permute(hidden_states, gate_weight, top_k)


def fused_gate_topk_ex(hidden_states, gate_weight, top_k, bias=None, return_logits=False, return_probs=False):
    """[ids int32, weights fp32, counts int32, offsets int32, sorted_idx int32, positions int32
    (, logits fp32 [T, E]) (, probs fp32 [T, E])] -- positions is the inverse permutation of
    sorted_idx, probs the full softmax probabilities."""
    return extension().fused_gate_topk_ex(hidden_states, gate_weight, top_k, bias, return_logits, return_probs)


def quantize_w4(w, group_size):
    """w [..., N, K] -> (qweight uint8 [..., N, K/2], scales fp16 [..., N, K/group_size])."""
    return extension().quantize_w4(w, group_size)


def dequantize_w4(qweight, scales, group_size):
    """int4 -> bf16 [..., N, K]; bit-exact bf16_rn(q * s)."""
    return extension().dequantize_w4(qweight, scales, group_size)


def prepack_w4(qweight, scales, group_size, qweight_up=None, scales_up=None):
    """Canonical int4 [E, N, K/2] + scales -> the GEMM's streaming layout (scales embedded;
    paired with the up projection if given).  Returns one uint8 tensor."""
    return extension().prepack_w4(qweight, scales, group_size, qweight_up, scales_up)


def w4a16_grouped_gemm(input, packed, expert_offsets, num_experts, N, group_size,
                       epilogue=0, dest_rows=None, row_scale=None, out_rows=0, max_rows_per_expert=0,
                       segment_expert=None):
    """Grouped W4A16 GEMM over `num_experts` row segments (segment_expert maps segment -> weights)."""
    return extension().w4a16_grouped_gemm(input, packed, expert_offsets, num_experts, N,
                                          group_size, epilogue, dest_rows, row_scale, out_rows,
                                          max_rows_per_expert, segment_expert)


def combine_rows(rows, positions, weights, num_tokens, top_k, extra_rows=None, num_extra=0):
    """y[t] = sum_j weights[t,j] * rows[positions[t,j]] + sum_s extra_rows[s*T + t]."""
    return extension().combine_rows(rows, positions, weights, num_tokens, top_k, extra_rows, num_extra)


def moe_layer_w4a16(x, gate_weight, w13_packed, w2_packed, top_k, ffn_size, group_size, num_shared=0,
                    gate_bias=None):
    """[y bf16 [T, d], ids int32 [T, k], weights fp32 [T, k]]."""
    return extension().moe_layer_w4a16(x, gate_weight, w13_packed, w2_packed, top_k, ffn_size, group_size,
                                       num_shared, gate_bias)
