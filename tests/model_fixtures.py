"""Model-side fixtures shared by the host and GPU tests: a tiny Hugging Face Mixtral
checkpoint on disk, and modules with the attribute structure of light-moe's MoE blocks
(python/light_moe/model/moe_block.py: SparseMoEBlock :88-117, SparseMoEBlockFast :186-212)."""
import json
import os

import torch

from light_moe_b200 import loader


def make_mixtral_dir(path, L=2, E=4, d=64, F=128, k=2, shards=2, seed=0, dtype=torch.bfloat16):
    """A tiny Mixtral-format checkpoint: config.json, sharded safetensors with the MoE tensors
    plus unrelated attention / norm tensors, and the shard index."""
    os.makedirs(path, exist_ok=True)
    cfg = {"hidden_size": d, "intermediate_size": F, "num_local_experts": E, "num_experts_per_tok": k,
           "num_hidden_layers": L, "model_type": "mixtral"}
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f)
    g = torch.Generator().manual_seed(seed)
    tensors = {"model.embed_tokens.weight": torch.randn(16, d, generator=g).to(dtype)}
    ref = {}
    for li in range(L):
        pre = f"model.layers.{li}"
        tensors[f"{pre}.self_attn.q_proj.weight"] = torch.randn(d, d, generator=g).to(dtype)
        tensors[f"{pre}.input_layernorm.weight"] = torch.ones(d, dtype=dtype)
        gate = (torch.randn(E, d, generator=g) * 0.3).to(dtype)
        tensors[f"{pre}.block_sparse_moe.gate.weight"] = gate
        ref[li] = {"gate": gate, "w1": [], "w3": [], "w2": []}
        for e in range(E):
            for r, shape in (("w1", (F, d)), ("w3", (F, d)), ("w2", (d, F))):
                w = (torch.randn(*shape, generator=g) * 0.05).to(dtype)
                tensors[f"{pre}.block_sparse_moe.experts.{e}.{r}.weight"] = w
                ref[li][r].append(w)
    names = sorted(tensors)
    weight_map = {}
    for s in range(shards):
        part = {n: tensors[n] for i, n in enumerate(names) if i % shards == s}
        fname = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
        loader.write_safetensors(os.path.join(path, fname), part, {"format": "pt"})
        weight_map.update({n: fname for n in part})
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": weight_map}, f)
    return cfg, ref



class _Expert(torch.nn.Module):
    def __init__(self, d, F):
        super().__init__()
        self.gate_proj = torch.nn.Linear(d, F, bias=False)
        self.up_proj = torch.nn.Linear(d, F, bias=False)
        self.down_proj = torch.nn.Linear(F, d, bias=False)


class _Gate(torch.nn.Module):
    def __init__(self, d, E, k, bias=False):
        super().__init__()
        self.gate = torch.nn.Linear(d, E, bias=bias)
        self.top_k = k
        self.aux_loss_coef = 0.02


class SparseBlockLike(torch.nn.Module):
    """The attribute structure of SparseMoEBlock."""

    def __init__(self, d=64, F=128, E=4, k=2, bias=False):
        super().__init__()
        self.top_k = k
        self.gate = _Gate(d, E, k, bias)
        self.experts = torch.nn.ModuleList([_Expert(d, F) for _ in range(E)])


class _Grouped(torch.nn.Module):
    def __init__(self, E, fin, fout):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.randn(E, fout, fin))
        self.register_parameter("bias", None)


class FastBlockLike(torch.nn.Module):
    """The attribute structure of SparseMoEBlockFast."""

    def __init__(self, d=64, F=128, E=4, k=2):
        super().__init__()
        self.top_k = k
        self.gate = _Gate(d, E, k)
        self.gate_proj = _Grouped(E, d, F)
        self.up_proj = _Grouped(E, d, F)
        self.down_proj = _Grouped(E, F, d)
