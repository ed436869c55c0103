"""Generate the golden fixtures by running light-moe's own PyTorch reference.

Run in a container where the reference checkout exists:

    LIGHT_MOE_REF=/root/reference/python python tests/golden/make_golden.py

The reference cannot travel to the GPU machines, so its outputs are recorded here as small
``.npz`` fixtures (inputs + outputs) that ``tests/test_oracle.py`` replays against the CPU
oracle.  What each fixture pins:

* ``routing_*.npz``   -- ``light_moe.ops.moe_gate.top_k_routing`` (moe_gate.py:39-77), the
  ``MoEGate.forward`` counts (moe_gate.py:202-214) and ``load_balancing_loss``
  (moe_gate.py:80-122) on fp32 logits without exact ties.
* ``permute_*.npz``   -- ``light_moe.ops.grouped_gemm.permute_tokens`` / ``unpermute_tokens``
  (grouped_gemm.py:202-279): offsets, and per-expert segment contents (the reference sort is
  unstable, so segments are compared as sorted lists).
* ``block_*.npz``     -- ``light_moe.model.moe_block.SparseMoEBlock.forward`` (moe_block.py:119-169)
  and ``SparseMoEBlockFast.forward`` (moe_block.py:216-274) in fp32 with known weights.
* ``block_cfg1_summary.npz`` -- the same block at the CPU-layer workload (T=512, d=1024,
  ffn=2816, E=8, top-2, N(0, 0.02) weights, N(0, 1) inputs, numpy PCG64 seed 0); only the
  routing and output rows 0..15 plus whole-output checksums are stored, the inputs are
  regenerated from the seed.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from inputs import BLOCK_CASES, block_inputs, cfg1_inputs  # noqa: E402


def _import_reference():
    ref = os.environ.get("LIGHT_MOE_REF")
    if not ref:
        raise SystemExit("set LIGHT_MOE_REF to the reference checkout's python/ directory")
    if ref not in sys.path:
        sys.path.insert(0, ref)
    import torch  # noqa: F401
    from light_moe.ops.moe_gate import top_k_routing, MoEGate  # noqa: F401
    from light_moe.ops.grouped_gemm import permute_tokens, unpermute_tokens  # noqa: F401
    from light_moe.model.moe_block import SparseMoEBlock, SparseMoEBlockFast  # noqa: F401
    # light_moe.ops re-exports a function named grouped_gemm that shadows the submodule
    mg = sys.modules["light_moe.ops.moe_gate"]
    gg = sys.modules["light_moe.ops.grouped_gemm"]
    mb = sys.modules["light_moe.model.moe_block"]
    return mg, gg, mb


def _load_block(mb, torch, d, ffn, E, k, gate_w, w1, w3, w2, fast=False):
    cls = mb.SparseMoEBlockFast if fast else mb.SparseMoEBlock
    blk = cls(d, ffn, num_experts=E, top_k=k)
    blk.eval()
    with torch.no_grad():
        blk.gate.gate.weight.copy_(torch.from_numpy(gate_w))
        if fast:
            blk.gate_proj.weight.copy_(torch.from_numpy(w1))
            blk.up_proj.weight.copy_(torch.from_numpy(w3))
            blk.down_proj.weight.copy_(torch.from_numpy(w2))
        else:
            for e in range(E):
                blk.experts[e].gate_proj.weight.copy_(torch.from_numpy(w1[e]))
                blk.experts[e].up_proj.weight.copy_(torch.from_numpy(w3[e]))
                blk.experts[e].down_proj.weight.copy_(torch.from_numpy(w2[e]))
    return blk


def main():
    import torch
    mg, gg, mb = _import_reference()
    torch.manual_seed(0)
    out = {}

    # ---- routing on fp32 logits (no exact ties in continuous random data) ----
    for (T, E, k, scale, seed) in [(257, 8, 2, 1.0, 1), (300, 64, 6, 1.5, 2), (64, 16, 4, 0.3, 3),
                                   (33, 8, 1, 2.0, 4), (128, 8, 8, 1.0, 5)]:
        rng = np.random.default_rng(seed)
        logits = (rng.standard_normal((T, E)) * scale).astype(np.float32)
        lt = torch.from_numpy(logits).view(1, T, E)
        idx, w, probs = mg.top_k_routing(lt, k, normalize=True, training=False)
        counts = torch.zeros(E, dtype=torch.int64)
        for j in range(k):
            counts += torch.bincount(idx[:, :, j].flatten(), minlength=E)
        # the load-balancing loss of these routings (moe_gate.py:80-122)
        aux = mg.load_balancing_loss(probs, idx, E)
        np.savez_compressed(os.path.join(HERE, f"routing_T{T}_E{E}_k{k}.npz"),
                            logits=logits, ids=idx.view(T, k).numpy().astype(np.int32),
                            weights=w.view(T, k).numpy().astype(np.float32),
                            probs=probs.view(T, E).numpy().astype(np.float32),
                            counts=counts.numpy().astype(np.int64),
                            aux_loss=np.float32(aux.item()))
        out[f"routing_{T}_{E}_{k}"] = True

    # ---- permute / unpermute ----
    for (B, S, d, E, k, seed) in [(2, 8, 64, 4, 2, 11), (1, 100, 32, 8, 2, 12), (3, 7, 16, 64, 6, 13)]:
        g = torch.Generator().manual_seed(seed)
        hs = torch.randn(B, S, d, generator=g)
        ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(B * S)]).view(B, S, k)
        rw = torch.softmax(torch.randn(B, S, k, generator=g), dim=-1)
        perm, offs, rev = gg.permute_tokens(hs, ids, E)
        unperm = gg.unpermute_tokens(perm, rev, rw)
        # segment contents as sorted flat indices (the reference argsort is unstable)
        flat = ids.view(-1)
        sorted_idx = torch.argsort(rev)  # inverse of reverse == the sort permutation used
        np.savez_compressed(os.path.join(HERE, f"permute_B{B}_S{S}_E{E}_k{k}.npz"),
                            hidden=hs.numpy().astype(np.float32),
                            ids=ids.numpy().astype(np.int32), rw=rw.numpy().astype(np.float32),
                            offsets=offs.numpy().astype(np.int64),
                            sorted_idx=sorted_idx.numpy().astype(np.int64),
                            permuted=perm.numpy().astype(np.float32),
                            unpermuted=unperm.numpy().astype(np.float32),
                            flat_ids=flat.numpy().astype(np.int32))

    # ---- SparseMoEBlock / SparseMoEBlockFast at small shapes (inputs regenerated from seeds) ----
    for (T, d, ffn, E, k, seed) in BLOCK_CASES:
        x, gate_w, w1, w3, w2 = block_inputs(T, d, ffn, E, seed)
        blk = _load_block(mb, torch, d, ffn, E, k, gate_w, w1, w3, w2)
        fast = _load_block(mb, torch, d, ffn, E, k, gate_w, w1, w3, w2, fast=True)
        with torch.no_grad():
            xt = torch.from_numpy(x).view(1, T, d)
            y, _ = blk(xt)
            yf, _ = fast(xt)
            r = blk.gate(xt, return_aux_loss=False)
        np.savez_compressed(os.path.join(HERE, f"block_T{T}_d{d}_f{ffn}_E{E}_k{k}.npz"),
                            ids=r.expert_indices.view(T, k).numpy().astype(np.int32),
                            weights=r.routing_weights.view(T, k).numpy().astype(np.float32),
                            counts=r.expert_counts.numpy().astype(np.int64),
                            y=y.view(T, d).numpy(), y_fast=yf.view(T, d).numpy())

    # ---- the CPU-layer workload (config 1): summary only ----
    x, gate_w, w1, w3, w2 = cfg1_inputs()
    T, d = x.shape
    E, ffn = w1.shape[0], w1.shape[1]
    blk = _load_block(mb, torch, d, ffn, E, 2, gate_w, w1, w3, w2)
    with torch.no_grad():
        xt = torch.from_numpy(x).view(1, T, d)
        y, _ = blk(xt)
        r = blk.gate(xt, return_aux_loss=False)
    y = y.view(T, d).numpy()
    np.savez_compressed(os.path.join(HERE, "block_cfg1_summary.npz"),
                        ids=r.expert_indices.view(T, 2).numpy().astype(np.int32),
                        weights=r.routing_weights.view(T, 2).numpy().astype(np.float32),
                        counts=r.expert_counts.numpy().astype(np.int64),
                        y_rows=y[:16].copy(), y_sum=np.float64(y.astype(np.float64).sum()),
                        y_abs_sum=np.float64(np.abs(y.astype(np.float64)).sum()),
                        y_row_norms=np.linalg.norm(y.astype(np.float64), axis=1))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
