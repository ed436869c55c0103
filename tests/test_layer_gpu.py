"""GPU parity of the whole W4A16 MoE layer.

The reference computation is light-moe's SparseMoEBlock.forward on the dequantised int4
weights in fp32 (CPU oracle restatement for small shapes; the same math as a plain PyTorch
fp32 computation on the GPU for the large ones), using the layer's own routing so that
near-tie routing flips do not enter the comparison; the routing itself is checked
separately against the oracle.  Bar: max |y - y_ref| / max |y_ref| <= 1e-2.
"""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import dequantize, layer
from light_moe_b200.layer import W4A16Experts, W4A16MoELayer

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _make(T, d, F, E, k, g, seed, S=0, bias=False, wscale=0.02):
    gen = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(T, d, generator=gen).to(torch.bfloat16).cuda()
    gw = (torch.randn(E, d, generator=gen) * 0.02).to(torch.bfloat16).cuda()
    w1 = (torch.randn(E + S, F, d, generator=gen) * wscale).to(torch.bfloat16).cuda()
    w3 = (torch.randn(E + S, F, d, generator=gen) * wscale).to(torch.bfloat16).cuda()
    w2 = (torch.randn(E + S, d, F, generator=gen) * wscale).to(torch.bfloat16).cuda()
    shared = [(w1[E + s], w3[E + s], w2[E + s]) for s in range(S)] or None
    ex = W4A16Experts.from_dense(w1[:E], w3[:E], w2[:E], g, shared=shared, keep_canonical=True)
    b = (torch.linspace(-1.0, 1.0, E, device="cuda") if bias else None)
    return x, gw, ex, b


def _deq(ex):
    c = ex.canonical
    g = ex.group_size
    return (dequantize(c["q1"], c["s1"], g).float(), dequantize(c["q3"], c["s3"], g).float(),
            dequantize(c["q2"], c["s2"], g).float())


def _ref_torch(x, ids, wts, d1, d3, d2, E):
    """SparseMoEBlock.forward restated in fp32 torch (moe_block.py:146-164)."""
    xf = x.float()
    out = torch.zeros_like(xf)
    ids = ids.long()
    for j in range(ids.shape[1]):
        for e in range(E):
            m = ids[:, j] == e
            if not m.any():
                continue
            xe = xf[m]
            h = torch.nn.functional.silu(xe @ d1[e].T) * (xe @ d3[e].T)
            out[m] += (h @ d2[e].T) * wts[m, j][:, None]
    for s in range(E, d1.shape[0]):
        h = torch.nn.functional.silu(xf @ d1[s].T) * (xf @ d3[s].T)
        out += h @ d2[s].T
    return out


def _check(y, ref):
    err = (y.float() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= TOL * scale, f"max rel err {err / scale:.3e}"


@pytest.mark.parametrize("T,d,F,E,k,g", [(64, 256, 256, 8, 2, 128), (200, 128, 256, 16, 4, 64), (5, 256, 256, 8, 2, 128)])
def test_layer_matches_cpu_oracle(T, d, F, E, k, g):
    x, gw, ex, _ = _make(T, d, F, E, k, g, seed=T)
    y, ids, wts = layer(x, gw, ex, k)
    d1, d3, d2 = _deq(ex)
    ids_np, w_np = ids.cpu().numpy(), wts.cpu().numpy()
    y_ref = oracle.reference_block_forward(x.float().cpu().numpy(), ids_np, w_np, d1.cpu().numpy(),
                                           d3.cpu().numpy(), d2.cpu().numpy())
    err = np.abs(y.float().cpu().numpy() - y_ref).max()
    assert err <= TOL * np.abs(y_ref).max()
    # routing: the oracle on the fp64 logits picks the same experts for well-separated tokens
    lg = oracle.gate_logits_f64(x.float().cpu().numpy(), gw.float().cpu().numpy())
    ref_ids, _ = oracle.route(lg.astype(np.float32), k)
    agree = (np.sort(ref_ids, 1) == np.sort(ids_np, 1)).all(1).mean()
    assert agree >= 0.97


def test_layer_module_and_shared_experts():
    T, d, F, E, k, g, S = 300, 256, 128, 16, 4, 64, 2
    x, gw, ex, b = _make(T, d, F, E, k, g, seed=1, S=S, bias=True)
    mod = W4A16MoELayer(gw, ex, k, gate_bias=b)
    y, ids, wts = mod(x, return_routing=True)
    d1, d3, d2 = _deq(ex)
    _check(y, _ref_torch(x, ids, wts, d1, d3, d2, E))


@pytest.mark.parametrize("T", [64, 8192])
def test_layer_mixtral_shape(T):
    """Mixtral-8x7B expert shapes (d=4096, ffn=14336, 8 experts top-2, g=128): decode and prefill."""
    d, F, E, k, g = 4096, 14336, 8, 2, 128
    x, gw, ex, _ = _make(T, d, F, E, k, g, seed=T)
    y, ids, wts = layer(x, gw, ex, k)
    d1, d3, d2 = _deq(ex)
    if T > 1024:
        # every 8th token (1024 of them, spread over the whole batch and so over every
        # expert segment and GEMM tile) keeps the fp32 reference cheap
        sl = slice(0, T, 8)
        assert torch.unique(ids[sl]).numel() == E
        _check(y[sl], _ref_torch(x[sl], ids[sl], wts[sl], d1, d3, d2, E))
    else:
        _check(y, _ref_torch(x, ids, wts, d1, d3, d2, E))


@pytest.mark.parametrize("T", [64, 2048])
def test_layer_fine_grained_shape(T):
    """64 routed experts (ffn 1408) top-6 + 2 shared, g=64, biased router; T=64 runs the
    decode kernels with two scale groups per 128-K stage."""
    d, F, E, k, g, S = 2048, 1408, 64, 6, 64, 2
    x, gw, ex, b = _make(T, d, F, E, k, g, seed=2, S=S, bias=True)
    mod = W4A16MoELayer(gw, ex, k, gate_bias=b)
    y, ids, wts = mod(x, return_routing=True)
    d1, d3, d2 = _deq(ex)
    _check(y, _ref_torch(x, ids, wts, d1, d3, d2, E))


@pytest.mark.parametrize("T,chunks", [(50, 4), (300, 3), (1000, 4), (1000, 16), (4097, 4), (129, 2), (258, 2)])
def test_forward_host_matches_forward(T, chunks):
    """Host-buffer layer call (chunked, copies overlapped with the kernels) == device call."""
    d, F, E, k, g = 256, 256, 8, 2, 128
    x, gw, ex, _ = _make(T, d, F, E, k, g, seed=3 + T)
    mod = W4A16MoELayer(gw, ex, k)
    y_dev = mod(x).cpu()
    xh = x.cpu().pin_memory()
    yh = mod.forward_host(xh, chunks=chunks)
    torch.cuda.synchronize()
    assert yh.is_pinned()
    assert torch.equal(yh.view(torch.int16), y_dev.view(torch.int16))
    # caller-provided output buffer, 3-D activations
    out = torch.empty((1, T, d), dtype=torch.bfloat16).pin_memory()
    mod.forward_host(xh.view(1, T, d), out=out, chunks=chunks)
    torch.cuda.synchronize()
    assert torch.equal(out.view(T, d).view(torch.int16), y_dev.view(torch.int16))
    with pytest.raises(ValueError):
        mod.forward_host(x, chunks=chunks)   # device input belongs to forward


def test_forward_host_async_back_to_back_calls():
    """Consecutive host-buffer calls without waiting in between (the next call's input copies
    beside this call's kernels, this call's output copies beside the next call's kernels):
    each output equals the device call on its own input, also when two calls share one
    output buffer and the first result is read before the second call overwrites it."""
    d, F, E, k, g = 256, 256, 8, 2, 128
    T = 3000
    xs, refs = [], []
    x0, gw, ex, _ = _make(T, d, F, E, k, g, seed=11)
    mod = W4A16MoELayer(gw, ex, k)
    for i in range(3):
        x = x0 if i == 0 else torch.randn(T, d, generator=torch.Generator().manual_seed(50 + i)).to(
            torch.bfloat16).cuda()
        xs.append(x.cpu().pin_memory())
        refs.append(mod(x).cpu())
    outs = [torch.empty(T, d, dtype=torch.bfloat16).pin_memory() for _ in range(3)]
    events = [mod.forward_host_async(xs[i], out=outs[i], chunks=3)[1] for i in range(3)]
    for i in range(3):
        events[i].synchronize()
        assert torch.equal(outs[i].view(torch.int16), refs[i].view(torch.int16)), i
    # one shared output buffer: the stream order keeps each result until the next call's copy
    shared = torch.empty(T, d, dtype=torch.bfloat16).pin_memory()
    _, ev = mod.forward_host_async(xs[1], out=shared, chunks=3)
    ev.synchronize()
    first = shared.clone()
    _, ev = mod.forward_host_async(xs[2], out=shared, chunks=3)
    ev.synchronize()
    assert torch.equal(first.view(torch.int16), refs[1].view(torch.int16))
    assert torch.equal(shared.view(torch.int16), refs[2].view(torch.int16))
