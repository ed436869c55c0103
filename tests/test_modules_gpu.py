"""GPU tests of the model-facing modules: the MoEGate router module (router_probs bit-exact,
load-balancing loss), the W4A16 block converted from both light-moe block layouts, the
model-level switch, and loading a Mixtral checkpoint into int4 layers (and back from the int4
file).  Layer outputs are checked against fp32 math on the dequantised weights with the
layer's own routing (max |y - y_ref| / max |y_ref| <= 1e-2)."""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import dequantize
from light_moe_b200 import integration, loader, ops
from light_moe_b200.router import MoEGate, load_balancing_loss
from model_fixtures import FastBlockLike, SparseBlockLike, make_mixtral_dir

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _ref_block(x, ids, wts, d1, d3, d2):
    xf = x.float()
    out = torch.zeros_like(xf)
    for j in range(ids.shape[1]):
        for e in range(d1.shape[0]):
            m = ids[:, j].long() == e
            if m.any():
                xe = xf[m]
                out[m] += (torch.nn.functional.silu(xe @ d1[e].T) * (xe @ d3[e].T)) @ d2[e].T * wts[m, j][:, None]
    return out


def _deq(ex):
    c, g = ex.canonical, ex.group_size
    return [dequantize(c[q], c[s], g).float() for q, s in (("q1", "s1"), ("q3", "s3"), ("q2", "s2"))]


def _check(y, ref):
    err = (y.float() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= TOL * scale, f"max rel err {err / scale:.3e}"


@pytest.mark.parametrize("T,d,E,k", [(100, 256, 8, 2), (3000, 512, 64, 6)])
def test_router_probabilities_bitexact(T, d, E, k):
    g = torch.Generator(device="cpu").manual_seed(T)
    x = torch.randn(T, d, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(E, d, generator=g) * 0.05).to(torch.bfloat16).cuda()
    ids, wts, counts, offs, sidx, pos, logits, probs = ops.fused_gate_topk_ex(x, w, k, None, True, True)
    want = oracle.softmax_probs(logits.cpu().numpy())
    assert np.array_equal(probs.cpu().numpy().view(np.uint32), want.view(np.uint32))
    ids_o, w_o = oracle.route(logits.cpu().numpy(), k)
    assert np.array_equal(ids.cpu().numpy(), ids_o)


def test_moe_gate_module():
    T, d, E, k = 2, 64, 8, 2
    gate = MoEGate(256, E, top_k=k, bias=True).cuda().to(torch.bfloat16)
    with torch.no_grad():
        gate.gate.bias.copy_(torch.linspace(-0.5, 0.5, E))
    x = torch.randn(T, d, 256, device="cuda").to(torch.bfloat16)
    gate.eval()
    out = gate(x)
    assert out.expert_indices.shape == (T, d, k) and out.expert_indices.dtype == torch.int64
    assert out.routing_weights.dtype == torch.bfloat16 and out.router_probs.shape == (T, d, E)
    assert out.aux_loss is None
    assert torch.equal(out.expert_counts, torch.bincount(out.expert_indices.flatten(), minlength=E))
    torch.testing.assert_close(out.routing_weights.float().sum(-1), torch.ones(T, d, device="cuda"), atol=1e-2, rtol=0)
    gate.train()
    out = gate(x)
    want = load_balancing_loss(out.router_probs.float(), out.expert_indices, E) * gate.aux_loss_coef
    torch.testing.assert_close(out.aux_loss.float(), want.float(), rtol=1e-2, atol=1e-4)


@pytest.mark.parametrize("layout", ["sparse", "fast"])
def test_block_conversion(layout):
    torch.manual_seed(3)
    d, F, E, k = 256, 256, 8, 2
    blk = (SparseBlockLike(d, F, E, k) if layout == "sparse" else FastBlockLike(d, F, E, k))
    with torch.no_grad():
        for p in blk.parameters():
            p.mul_(0.05 if p.dim() == 3 else 1.0)
    blk = blk.to(torch.bfloat16)
    mod = integration.SparseMoEBlockW4A16.from_block(blk.eval(), group_size=128)
    assert not mod.training
    x = torch.randn(3, 40, d, device="cuda").to(torch.bfloat16)
    y, aux = mod(x)
    assert y.shape == x.shape and y.dtype == x.dtype and aux is None
    # the same routing and the dequantised int4 experts, in fp32
    ex = integration.block_weights(blk)
    q = {r: ops.quantize_w4(ex[r].cuda(), 128) for r in ("w1", "w3", "w2")}
    deq = [dequantize(*q[r], 128).float() for r in ("w1", "w3", "w2")]
    x2 = x.reshape(-1, d)
    ids, wts = ops.fused_gate_topk_ex(x2, ex["gate"].cuda(), k)[:2]
    _check(y.reshape(-1, d), _ref_block(x2, ids, wts, *deq))
    # fp32 activations in, fp32 out
    y32, _ = mod(x.float())
    assert y32.dtype == torch.float32
    mod.train()
    _, aux = mod(x)
    assert aux is not None and aux.numel() == 1


def test_enable_w4a16_on_a_model():
    class Layer(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.moe = SparseBlockLike(128, 128, 4, 2).to(torch.bfloat16)

    model = torch.nn.ModuleList([Layer(), Layer()])
    assert integration.enable_w4a16(model) == 2
    x = torch.randn(1, 8, 128, device="cuda").to(torch.bfloat16)
    for layer in model:
        assert isinstance(layer.moe, integration.SparseMoEBlockW4A16)
        y, aux = layer.moe(x)
        assert y.shape == x.shape and torch.isfinite(y.float()).all()


def test_mixtral_checkpoint_to_int4_file_and_back(tmp_path):
    ckpt = str(tmp_path / "mixtral")
    make_mixtral_dir(ckpt, L=2, E=4, d=256, F=256, k=2, shards=2)
    meta = loader.quantize_hf_mixtral(ckpt, str(tmp_path / "w4.safetensors"), group_size=128)
    assert meta["layers"] == "0,1" and meta["group_size"] == "128"
    from_file = loader.load_w4a16(str(tmp_path / "w4.safetensors"))
    direct = loader.load_hf_mixtral_moe(ckpt, group_size=128)
    x = torch.randn(50, 256, device="cuda").to(torch.bfloat16)
    for li in (0, 1):
        y1, ids, wts = from_file[li](x, return_routing=True)
        y2 = direct[li](x)
        assert torch.equal(y1, y2)
        _check(y1, _ref_block(x, ids, wts, *_deq(from_file[li].experts)))
    # re-saving the directly loaded layers gives the same int4 tensors
    loader.save_w4a16(str(tmp_path / "again.safetensors"), direct)
    with loader.SafetensorsFile(str(tmp_path / "w4.safetensors")) as a, \
            loader.SafetensorsFile(str(tmp_path / "again.safetensors")) as b:
        assert sorted(a.keys()) == sorted(b.keys())
        for n in a.keys():
            assert torch.equal(a.get(n), b.get(n)), n
