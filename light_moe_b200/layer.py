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

# Batches of at most this many tokens take other kernels than larger ones: the CUDA-core
# router (csrc/router.cu, kSmallTokens = 128; its fp32 dot products round differently from
# the tensor-core logits) and, at 64 tokens or fewer, the decode GEMMs (csrc/layer.cu).
SMALL_BATCH_TOKENS = 128


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


class HostBufferCalls:
    """forward_host / forward_host_async for a layer module whose ``forward`` runs on the
    device of ``self.gate_weight``: host-resident activations in, host-resident outputs out,
    the PCIe copies on two copy streams beside the kernels.  ``_host_ranges`` False keeps
    every call one token range (a layer whose ranks must all run the same number of steps)."""

    _host_ranges = True

    def forward_host(self, x_host: torch.Tensor, out: Optional[torch.Tensor] = None,
                     chunks: Optional[int] = None) -> torch.Tensor:
        """The layer on host-resident activations: x_host [..., d] bf16 on the CPU (pinned for
        asynchronous copies) in, y written to ``out`` (pinned host [..., d], allocated if None).

        The tokens are split into ``chunks`` contiguous ranges (default: one per 2560 tokens,
        at most 4: smaller ranges leave the GEMMs' 192-token tiles partly empty, which costs
        more than the copies they hide); the host-to-device copy of
        range c + 1 and the device-to-host copy of range c - 1 run on copy streams while
        range c is computed, so the PCIe transfers hide behind the kernels.  Every token's
        output depends on that token alone and every range keeps more than
        ``SMALL_BATCH_TOKENS`` tokens (a batch that small is one range), so each range runs
        the same kernels as the whole batch would and the result is bit-identical to
        ``forward(x_host.cuda()).cpu()``.  Returns ``out``; it is complete once the current
        CUDA stream has reached the point of return (synchronise before reading it).  The
        input copies of a call start at once, beside the previous call's kernels.
        """
        if chunks is None:   # one call on its own: hide the copies behind its own token ranges
            chunks = min(4, x_host.reshape(-1, x_host.shape[-1]).shape[0] // 2560) if self._host_ranges else 1
        out, done = self.forward_host_async(x_host, out, chunks)
        if done is not None:
            torch.cuda.current_stream(self.gate_weight.device).wait_event(done)
        return out

    def forward_host_async(self, x_host: torch.Tensor, out: Optional[torch.Tensor] = None,
                           chunks: int = 1):
        """forward_host without the current stream waiting for the output copies: returns
        (out, done), ``done`` a CUDA event recorded after the last device-to-host copy
        (``done.synchronize()``, or make a stream wait on it, before reading ``out``; None for
        an empty batch).  In a
        loop of calls the output copies of one call overlap the next call's kernels, and its
        input copies the previous call's kernels; calls keep their order on every stream, so
        consecutive calls may reuse the same ``out`` and ``x_host``.  Same results as
        forward_host.  ``chunks`` defaults to one token range: in a loop of calls the
        neighbouring calls' kernels already hide the copies, and whole-batch GEMM tiles are
        fuller (8192 tokens of the Mixtral layer: 5.42-5.50 ms per call against 5.78-5.86
        with 2-3 ranges, 5.24 ms device-only)."""
        if not self._host_ranges and chunks != 1:
            raise ValueError("this layer runs every call as one token range (chunks=1)")
        if x_host.device.type != "cpu":
            raise ValueError("forward_host takes host activations; use forward for device tensors")
        if x_host.dtype != torch.bfloat16:
            raise ValueError("activations must be bf16")
        shape = x_host.shape
        x2 = x_host.reshape(-1, shape[-1])
        if out is None:
            out = torch.empty(shape, dtype=torch.bfloat16, pin_memory=True)
        elif out.shape != shape or out.dtype != torch.bfloat16 or out.device.type != "cpu":
            raise ValueError("out must be a bf16 host tensor shaped like x_host")
        if not out.is_contiguous():
            raise ValueError("out must be contiguous")
        y2 = out.view(-1, shape[-1])
        T = x2.shape[0]
        if T == 0 and self._host_ranges:
            return out, None   # nothing to copy or compute (a multi-rank layer still takes its step)
        device = self.gate_weight.device
        cur = torch.cuda.current_stream(device)
        if not hasattr(self, "_copy_streams"):
            self._copy_streams = (torch.cuda.Stream(device), torch.cuda.Stream(device))
        h2d, d2h = self._copy_streams
        done = torch.cuda.Event()
        n = 1 if T <= SMALL_BATCH_TOKENS else max(1, min(int(chunks), T // (SMALL_BATCH_TOKENS + 1)))
        bounds = [T * i // n for i in range(n + 1)]
        loaded = []
        with torch.cuda.stream(h2d):
            # the staging buffer belongs to the copy stream (its memory is free there), so the
            # copies start without waiting for the current stream's earlier work
            xd = torch.empty((T, shape[-1]), dtype=torch.bfloat16, device=device)
            for i in range(n):
                a, b = bounds[i], bounds[i + 1]
                xd[a:b].copy_(x2[a:b], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(h2d)
                loaded.append(ev)
        xd.record_stream(cur)
        for i in range(n):
            a, b = bounds[i], bounds[i + 1]
            cur.wait_event(loaded[i])
            yc = self.forward(xd[a:b])
            d2h.wait_stream(cur)
            with torch.cuda.stream(d2h):
                y2[a:b].copy_(yc, non_blocking=True)
            yc.record_stream(d2h)
        done.record(d2h)
        return out, done


class W4A16MoELayer(HostBufferCalls, torch.nn.Module):
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

