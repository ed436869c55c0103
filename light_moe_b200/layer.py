"""W4A16 MoE layer module.

``W4A16Experts`` holds the int4 expert weights in the GEMM's streaming layout;
``W4A16MoELayer`` is the drop-in counterpart of light-moe's ``SparseMoEBlock``
(python/light_moe/model/moe_block.py:63-169): same routing (bias-free Linear(d, E) router
by default, softmax -> top-k -> renormalise) and the same SwiGLU experts
``down(silu(gate(x)) * up(x))`` with the Mixtral roles w1 = gate, w3 = up, w2 = down
(python/light_moe/model/loader.py:123-128), but with int4 expert weights and the whole
layer running in one stream of sm_100a kernels.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Sequence, Tuple

import torch

from . import ops


@dataclass
class W4A16Experts:
    """Prepacked int4 experts: ``num_experts`` routed experts followed by ``num_shared``."""

    w13_packed: torch.Tensor   # paired gate/up super-blocks, scales embedded
    w2_packed: torch.Tensor    # down super-blocks, scales embedded
    num_experts: int
    num_shared: int
    hidden_size: int
    ffn_size: int
    group_size: int
    # canonical copies (kept for checking / saving); optional
    canonical: Optional[dict] = None

    @classmethod
    def from_dense(cls, w1: torch.Tensor, w3: torch.Tensor, w2: torch.Tensor, group_size: int,
                   shared: Optional[Sequence[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]]] = None,
                   keep_canonical: bool = False) -> "W4A16Experts":
        """Quantise dense expert weights on the GPU and prepack them.

        w1, w3: [E, ffn, d] (gate, up); w2: [E, d, ffn]; ``shared``: list of (w1, w3, w2) with
        shapes [ffn, d], [ffn, d], [d, ffn] for always-on experts.
        """
        E, F, d = w1.shape
        if shared:
            w1 = torch.cat([w1] + [s[0].unsqueeze(0) for s in shared])
            w3 = torch.cat([w3] + [s[1].unsqueeze(0) for s in shared])
            w2 = torch.cat([w2] + [s[2].unsqueeze(0) for s in shared])
        q1, s1 = ops.quantize_w4(w1, group_size)
        q3, s3 = ops.quantize_w4(w3, group_size)
        q2, s2 = ops.quantize_w4(w2, group_size)
        return cls.from_quantized(q1, s1, q3, s3, q2, s2, E, group_size, keep_canonical=keep_canonical)

    @classmethod
    def from_quantized(cls, q1, s1, q3, s3, q2, s2, num_experts: int, group_size: int,
                       keep_canonical: bool = False) -> "W4A16Experts":
        """From canonical int4 tensors (routed experts first, then shared ones)."""
        Et, F, d2 = q1.shape
        d = d2 * 2
        w13p = ops.prepack_w4(q1, s1, group_size, q3, s3)
        w2p = ops.prepack_w4(q2, s2, group_size)
        canon = dict(q1=q1, s1=s1, q3=q3, s3=s3, q2=q2, s2=s2) if keep_canonical else None
        return cls(w13p, w2p, num_experts, Et - num_experts, d, F, group_size, canon)


class W4A16MoELayer(torch.nn.Module):
    """y = sum_j w_j * expert_{e_j}(x)  (+ shared experts), int4 experts, bf16 activations."""

    def __init__(self, gate_weight: torch.Tensor, experts: W4A16Experts, top_k: int,
                 gate_bias: Optional[torch.Tensor] = None):
        super().__init__()
        if gate_weight.shape != (experts.num_experts, experts.hidden_size):
            raise ValueError("gate_weight must be [num_experts, hidden_size]")
        self.register_buffer("gate_weight", gate_weight.to(torch.bfloat16).contiguous())
        self.register_buffer("gate_bias", None if gate_bias is None else gate_bias.float().contiguous())
        self.experts = experts
        self.top_k = int(top_k)

    def forward(self, x: torch.Tensor, return_routing: bool = False):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        e = self.experts
        y, ids, w = ops.moe_layer_w4a16(x2, self.gate_weight, e.w13_packed, e.w2_packed, self.top_k,
                                        e.ffn_size, e.group_size, e.num_shared, self.gate_bias)
        y = y.view(*shape[:-1], shape[-1])
        return (y, ids, w) if return_routing else y
