"""numpy restatement of light-moe's MoE layer (test infrastructure only).

``reference_block_forward`` follows ``SparseMoEBlock.forward``
(python/light_moe/model/moe_block.py:119-169) step for step: route, then for every slot j
and every expert e gather the tokens whose j-th choice is e, run the SwiGLU expert
``down(silu(gate(x)) * up(x))`` (moe_block.py:50-60 with swiglu from
python/light_moe/ops/activation.py:30-50) and accumulate ``y * w`` in fp32.

All arithmetic is fp32 numpy (BLAS matmuls), as the reference's CPU path is fp32 torch.
"""
from __future__ import annotations

import numpy as np

from . import core


def gate_logits_f64(x, gate_w, gate_bias=None) -> np.ndarray:
    """fp64 router logits x @ W^T (+ b) -- the high-precision reference for the fp32 kernel."""
    lg = np.asarray(x, np.float64) @ np.asarray(gate_w, np.float64).T
    if gate_bias is not None:
        lg = lg + np.asarray(gate_bias, np.float64)[None, :]
    return lg


def _silu(g: np.ndarray) -> np.ndarray:
    return g / (np.float32(1.0) + np.exp(-g))


def expert_mlp_ref(x, w1, w3, w2) -> np.ndarray:
    """down(silu(gate(x)) * up(x)); w1 = gate [ffn, d], w3 = up [ffn, d], w2 = down [d, ffn]."""
    x = np.asarray(x, np.float32)
    g = x @ np.asarray(w1, np.float32).T
    u = x @ np.asarray(w3, np.float32).T
    h = _silu(g) * u
    return h @ np.asarray(w2, np.float32).T


def reference_block_forward(x, ids, weights, w1, w3, w2, shared=None) -> np.ndarray:
    """Restatement of SparseMoEBlock.forward given the routing (moe_block.py:134-169).

    x [T, d]; ids / weights [T, k]; w1, w3 [E, ffn, d]; w2 [E, d, ffn] (fp32 values, e.g.
    the dequantised int4 weights).  ``shared``: optional list of (w1, w3, w2) always-on
    experts added with weight 1.
    """
    x = np.asarray(x, np.float32)
    T, d = x.shape
    k = ids.shape[1]
    E = w1.shape[0]
    out = np.zeros((T, d), np.float32)
    for j in range(k):
        ej = ids[:, j]
        wj = np.asarray(weights[:, j], np.float32)
        for e in range(E):
            mask = ej == e
            if not mask.any():
                continue
            ye = expert_mlp_ref(x[mask], w1[e], w3[e], w2[e])
            out[mask] += ye * wj[mask][:, None]
    if shared:
        for (s1, s3, s2) in shared:
            out += expert_mlp_ref(x, s1, s3, s2)
    return out


def moe_layer_ref(x, gate_w, w1, w3, w2, top_k, gate_bias=None, shared=None, routing=None):
    """Full layer oracle: fp32 logits -> oracle routing -> block forward.

    ``routing`` = (ids, weights) overrides the oracle routing (used to compare the layer
    math with the GPU's own routing so that near-tie flips do not enter the comparison).
    Returns (y [T, d] fp32, ids, weights).
    """
    if routing is None:
        lg = (np.asarray(x, np.float32) @ np.asarray(gate_w, np.float32).T)
        if gate_bias is not None:
            lg = lg + np.asarray(gate_bias, np.float32)[None, :]
        ids, weights = core.route(lg.astype(np.float32), top_k)
    else:
        ids, weights = routing
    y = reference_block_forward(x, ids, weights, w1, w3, w2, shared=shared)
    return y, ids, weights
