"""Putting the W4A16 layer into light-moe's model: block conversion and a model-level switch.

light-moe builds every transformer block's feed-forward part as
``self.moe = SparseMoEBlock(hidden_size, intermediate_size, num_experts, top_k)``
(python/light_moe/model/transformer.py:57-62) and calls ``output, aux_loss = self.moe(x)``.
Two block layouts exist (python/light_moe/model/moe_block.py):

* ``SparseMoEBlock`` (:63-169): ``gate.gate`` = ``nn.Linear(d, E)`` router and
  ``experts[e].{gate_proj, up_proj, down_proj}`` ``nn.Linear`` experts (SwiGLU,
  ``down(silu(gate(x)) * up(x))``, :50-60);
* ``SparseMoEBlockFast`` (:179-274): the same router and ``GroupedLinear`` projections
  ``gate_proj / up_proj`` ``[E, ffn, d]`` and ``down_proj`` ``[E, d, ffn]``.

``SparseMoEBlockW4A16`` takes the place of either: same call signature
(``[batch, seq, d] -> (output, aux_loss)``), same routing (softmax -> top-k -> renormalise,
lower expert id on ties), the experts quantised to int4 (symmetric, per group of
``group_size`` input values, fp16 scales) and the whole block running as the library's
sm_100a kernels.  ``enable_w4a16(model)`` converts every block of a model in place -- the
flag that switches a model built from the reference's modules onto this path.
"""
from __future__ import annotations

from typing import Optional

import torch

from .layer import W4A16Experts, W4A16MoELayer
from .router import MoEGate, load_balancing_loss


def _linear_weight(mod) -> torch.Tensor:
    w = getattr(mod, "weight", None)
    if w is None:
        raise TypeError(f"{type(mod).__name__} has no weight")
    if getattr(mod, "bias", None) is not None:
        raise ValueError("expert projections with a bias are not supported by the W4A16 experts")
    return w.detach()


def block_weights(block) -> dict:
    """The router and expert weights of a light-moe MoE block, in the Mixtral roles
    w1 = gate_proj, w3 = up_proj, w2 = down_proj (python/light_moe/model/loader.py:123-128):
    ``{"gate": [E, d], "gate_bias": [E] or None, "w1": [E, ffn, d], "w3": [E, ffn, d],
    "w2": [E, d, ffn], "top_k": k, "aux_loss_coef": c}``.

    Accepts the ``SparseMoEBlock`` layout (``experts`` ModuleList of ``MoEExpert``) and the
    ``SparseMoEBlockFast`` layout (``GroupedLinear`` ``gate_proj / up_proj / down_proj``).
    """
    gate = block.gate
    router = gate.gate if hasattr(gate, "gate") else gate
    gw = router.weight.detach()
    gb = router.bias.detach() if getattr(router, "bias", None) is not None else None
    if hasattr(block, "experts"):
        experts = list(block.experts)
        w1 = torch.stack([_linear_weight(e.gate_proj) for e in experts])
        w3 = torch.stack([_linear_weight(e.up_proj) for e in experts])
        w2 = torch.stack([_linear_weight(e.down_proj) for e in experts])
    elif hasattr(block, "gate_proj"):
        for name in ("gate_proj", "up_proj", "down_proj"):
            if getattr(getattr(block, name), "bias", None) is not None:
                raise ValueError("expert projections with a bias are not supported by the W4A16 experts")
        w1 = block.gate_proj.weight.detach()
        w3 = block.up_proj.weight.detach()
        w2 = block.down_proj.weight.detach()
    else:
        raise TypeError(f"{type(block).__name__} is not a light-moe MoE block")
    E, F, d = w1.shape
    if gw.shape != (E, d) or w3.shape != (E, F, d) or w2.shape != (E, d, F):
        raise ValueError("inconsistent router / expert shapes")
    top_k = int(getattr(block, "top_k", getattr(gate, "top_k", 2)))
    coef = float(getattr(gate, "aux_loss_coef", 0.01))
    return {"gate": gw, "gate_bias": gb, "w1": w1, "w3": w3, "w2": w2, "top_k": top_k, "aux_loss_coef": coef}


class SparseMoEBlockW4A16(torch.nn.Module):
    """Drop-in for ``SparseMoEBlock`` / ``SparseMoEBlockFast`` with int4 experts.

    ``forward(hidden_states [batch, seq, d]) -> (output [batch, seq, d], aux_loss)``, like
    the reference block (moe_block.py:119-169).  The activations run in bf16 (inputs of other
    dtypes are converted; the output has the input's dtype); ``aux_loss`` is the load-balancing
    loss (moe_gate.py:80-122) times ``aux_loss_coef`` in training mode and None otherwise,
    as in ``MoEGate.forward`` (moe_gate.py:216-221).
    """

    def __init__(self, gate_weight: torch.Tensor, experts: W4A16Experts, top_k: int,
                 gate_bias: Optional[torch.Tensor] = None, aux_loss_coef: float = 0.01):
        super().__init__()
        self.layer = W4A16MoELayer(gate_weight, experts, top_k, gate_bias=gate_bias)
        self.hidden_size = experts.hidden_size
        self.intermediate_size = experts.ffn_size
        self.num_experts = experts.num_experts
        self.top_k = int(top_k)
        self.aux_loss_coef = float(aux_loss_coef)

    @classmethod
    def from_block(cls, block, group_size: int = 128, device: Optional[torch.device] = None) -> "SparseMoEBlockW4A16":
        """Quantise a light-moe block's experts (on ``device``, default the current CUDA
        device) and build the W4A16 block with the same router."""
        wts = block_weights(block)
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        experts = W4A16Experts.from_dense(wts["w1"].to(dev), wts["w3"].to(dev), wts["w2"].to(dev), group_size)
        gb = wts["gate_bias"].to(dev) if wts["gate_bias"] is not None else None
        mod = cls(wts["gate"].to(dev), experts, wts["top_k"], gate_bias=gb, aux_loss_coef=wts["aux_loss_coef"])
        return mod.train(getattr(block, "training", False))

    def forward(self, hidden_states: torch.Tensor):
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1])
        xb = x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)
        aux = None
        if self.training:
            probs_gate = MoEGate.from_weights(self.layer.gate_weight, self.top_k, self.layer.gate_bias,
                                              self.aux_loss_coef)
            out = probs_gate(xb.view(1, *xb.shape), return_aux_loss=True)
            aux = out.aux_loss
        y = self.layer(xb)
        if y.dtype != hidden_states.dtype:
            y = y.to(hidden_states.dtype)
        return y.view(shape), aux


def convert_block(block, group_size: int = 128, device: Optional[torch.device] = None) -> SparseMoEBlockW4A16:
    """``SparseMoEBlockW4A16.from_block``."""
    return SparseMoEBlockW4A16.from_block(block, group_size=group_size, device=device)


def _is_moe_block(mod) -> bool:
    if isinstance(mod, SparseMoEBlockW4A16):
        return False
    has_router = hasattr(mod, "gate") and (hasattr(mod.gate, "gate") or hasattr(mod.gate, "weight"))
    return has_router and (hasattr(mod, "experts") or hasattr(mod, "gate_proj"))


def enable_w4a16(model: torch.nn.Module, group_size: int = 128, device: Optional[torch.device] = None) -> int:
    """Replace every light-moe MoE block inside ``model`` by its W4A16 counterpart, in place
    (the blocks light-moe assigns to ``TransformerBlock.moe``, transformer.py:57-62, and any
    other attribute holding one).  Returns the number of blocks converted."""
    todo = []
    for name, mod in model.named_modules():
        for child_name, child in mod.named_children():
            if _is_moe_block(child):
                todo.append((mod, child_name, child))
    for parent, child_name, child in todo:
        setattr(parent, child_name, convert_block(child, group_size=group_size, device=device))
    return len(todo)
