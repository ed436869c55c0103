"""The router as a module: light-moe's ``MoEGate`` interface on the fused sm_100a router.

Mirrors python/light_moe/ops/moe_gate.py of the reference:

* ``RoutingOutput`` (:20-36): expert indices, routing weights, per-expert counts, the full
  softmax probabilities ``router_probs`` and the auxiliary load-balancing loss;
* ``load_balancing_loss`` (:80-122): ``num_experts * sum_e f_e * P_e`` with ``f_e`` the
  fraction of tokens routed to expert e and ``P_e`` its mean routing probability;
* ``MoEGate`` (:125-228): ``gate = nn.Linear(hidden_size, num_experts, bias)``, the same
  parameter names (a reference state dict loads unchanged), ``forward(hidden_states
  [batch, seq, d], return_aux_loss=True) -> RoutingOutput``, the loss (times
  ``aux_loss_coef``) only in training mode.

Logits, softmax, top-k (ties to the lower expert id), renormalisation, the counts and the
probabilities all come from one router kernel call (``fused_gate_topk_ex`` with
``return_probs``); the loss itself is the reference formula on those outputs.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn.functional as F

from . import ops


@dataclass
class RoutingOutput:
    """Router outputs (moe_gate.py:20-36 of the reference)."""

    expert_indices: torch.Tensor                 # [batch, seq, top_k] int64
    routing_weights: torch.Tensor                # [batch, seq, top_k], the hidden states' dtype
    expert_counts: torch.Tensor                  # [num_experts] int64
    router_probs: Optional[torch.Tensor] = None  # [batch, seq, num_experts]
    aux_loss: Optional[torch.Tensor] = None


def load_balancing_loss(router_probs: torch.Tensor, expert_indices: torch.Tensor, num_experts: int) -> torch.Tensor:
    """``num_experts * sum_e f_e * P_e`` (moe_gate.py:80-122): f_e = tokens routed to e / tokens
    (each token counts once per selected expert), P_e = mean probability of e over tokens."""
    probs = router_probs.reshape(-1, num_experts)
    idx = expert_indices.reshape(-1, expert_indices.shape[-1]).long()
    num_tokens = probs.shape[0]
    tokens_per_expert = F.one_hot(idx, num_experts).sum(dim=1).float().sum(dim=0)
    return num_experts * (tokens_per_expert / num_tokens * probs.mean(dim=0)).sum()


class MoEGate(torch.nn.Module):
    """Router module with the reference's constructor and forward (moe_gate.py:151-228)."""

    def __init__(self, hidden_size: int, num_experts: int, top_k: int = 2, routing_type: str = "softmax",
                 jitter_noise: float = 0.0, aux_loss_coef: float = 0.01, bias: bool = False):
        super().__init__()
        if routing_type != "softmax":
            raise ValueError("only softmax routing is implemented (the reference's forward routes by softmax too)")
        self.hidden_size = hidden_size
        self.num_experts = num_experts
        self.top_k = top_k
        self.routing_type = routing_type
        self.jitter_noise = jitter_noise
        self.aux_loss_coef = aux_loss_coef
        self.gate = torch.nn.Linear(hidden_size, num_experts, bias=bias)

    @classmethod
    def from_weights(cls, weight: torch.Tensor, top_k: int, bias: Optional[torch.Tensor] = None,
                     aux_loss_coef: float = 0.01) -> "MoEGate":
        """A gate holding the given router weight [E, d] (and bias [E]) by reference."""
        E, d = weight.shape
        g = cls.__new__(cls)
        torch.nn.Module.__init__(g)
        g.hidden_size, g.num_experts, g.top_k = d, E, int(top_k)
        g.routing_type, g.jitter_noise, g.aux_loss_coef = "softmax", 0.0, float(aux_loss_coef)
        g.gate = torch.nn.Linear(d, E, bias=bias is not None, device=weight.device, dtype=weight.dtype)
        with torch.no_grad():
            g.gate.weight = torch.nn.Parameter(weight, requires_grad=False)
            if bias is not None:
                g.gate.bias = torch.nn.Parameter(bias, requires_grad=False)
        return g

    def forward(self, hidden_states: torch.Tensor, return_aux_loss: bool = True) -> RoutingOutput:
        if self.training and self.jitter_noise > 0:
            raise NotImplementedError("router jitter noise is not implemented by the fused router")
        lead = hidden_states.shape[:-1]
        x = hidden_states.reshape(-1, hidden_states.shape[-1])
        bias = self.gate.bias.detach().float() if self.gate.bias is not None else None
        ids, w, counts, _offsets, _sidx, _pos, probs = ops.fused_gate_topk_ex(
            x, self.gate.weight.detach(), self.top_k, bias, False, True)
        k, E = self.top_k, self.num_experts
        expert_indices = ids.long().view(*lead, k)
        routing_weights = w.to(hidden_states.dtype).view(*lead, k)
        router_probs = probs.to(hidden_states.dtype).view(*lead, E)
        aux = None
        if return_aux_loss and self.training:
            aux = load_balancing_loss(probs.view(*lead, E), expert_indices, E) * self.aux_loss_coef
        return RoutingOutput(expert_indices=expert_indices, routing_weights=routing_weights,
                             expert_counts=counts.long(), router_probs=router_probs, aux_loss=aux)

    def extra_repr(self) -> str:
        return f"hidden_size={self.hidden_size}, num_experts={self.num_experts}, top_k={self.top_k}"
