"""Expert-parallel W4A16 MoE layer over NCCL (one process per GPU).

Keeps the interface of light-moe's expert-parallel module
(python/light_moe/distributed/expert_parallel.py:17-87: ``ExpertParallelConfig``,
``ExpertParallelGroup``) and replaces its ``ExpertParallelMoELayer`` (:90-354), which pads
to equal splits and applies local expert 0 to every token, with the real computation:

  1. route the rank's own tokens (router kernel: ids, weights, counts, offsets, stable
     sorted order and its inverse) -- tokens are data-parallel, the router is replicated;
  2. gather the token rows in expert order; experts live in contiguous blocks per rank
     (rank r owns [r*E/ep, (r+1)*E/ep), as at expert_parallel.py:120-121), so this order
     is also destination-rank order;
  3. exchange the per-(rank, expert) counts with one all-to-all and copy them to the host
     (the only host synchronisation: NCCL needs the split sizes);
  4. all-to-all-v dispatch of the bf16 rows;
  5. the received rows are grouped by (source rank, local expert); the grouped GEMMs take
     those segments directly, with a segment -> expert map, so no local re-sort is needed:
     gate/up GEMM with the SwiGLU epilogue, then the down GEMM;
  6. all-to-all-v combine back to the source ranks (same split sizes, reversed);
  7. weighted combine into the token order with the inverse permutation (fp32, slot order);
     always-on shared experts run locally on the rank's tokens in the same GEMM launches.

With ``micro_batches`` > 1 (the same value on every rank: it fixes the sequence of
collectives) each rank's tokens are split into that many contiguous micro-batches, possibly
empty: all of them are routed and gathered first and their counts travel in one
all-to-all (one host synchronisation per forward); then the dispatch all-to-alls are
enqueued back to back on NCCL's stream while the GEMMs of micro-batch m run on the compute
stream, and the combine all-to-all of m overlaps the GEMMs of m + 1.  Each token's
arithmetic is unchanged.

With ``dispatch="capacity"`` (decode: small batches of at most ``capacity_tokens`` tokens
per rank, the same bound on every rank) nothing is copied to the host: every rank sends
every other rank a fixed block of C = capacity_tokens * top_k rows (its rows for that rank,
then padding), so both all-to-alls have equal, host-known splits; the per-(rank, expert)
counts still travel in a small all-to-all, but only the device reads them: the received
rows are regrouped expert-major by a device-computed permutation (so each local expert's
weights stream once), the segment offsets are prefix sums on the device, the padding of
all source ranks is one "hole" segment (weight matrix -1, skipped by the GEMMs), and the
combine reads the returned block through the padded positions of the rank's own sorted
rows.  The whole step can be captured in a
CUDA graph.  The reference pads to equal splits as well (expert_parallel.py:186-244) but
sends every token to every rank; here only the routed rows carry data.

The steps that move data between ranks use ``torch.distributed`` collectives, so the
whole flow also runs with the gloo backend on CPU processes when a CPU expert backend is
supplied (the tests do this); the product backend is the CUDA library.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from datetime import timedelta
from typing import Optional

import torch
import torch.distributed as dist

from . import ops
from .layer import HostBufferCalls, W4A16Experts


@dataclass
class ExpertParallelConfig:
    """Configuration for expert parallelism (expert_parallel.py:17-30 of the reference)."""

    num_experts: int = 8
    top_k: int = 2
    hidden_size: int = 4096
    intermediate_size: int = 14336
    ep_size: int = 8
    group_size: int = 128
    num_shared: int = 0

    @property
    def experts_per_rank(self) -> int:
        assert self.num_experts % self.ep_size == 0, "num_experts must be divisible by ep_size"
        return self.num_experts // self.ep_size


class ExpertParallelGroup:
    """The expert-parallel process group (expert_parallel.py:33-87 of the reference)."""

    def __init__(self, ep_size: int = 8):
        self.ep_size = ep_size
        self.group: Optional[dist.ProcessGroup] = None
        self.rank = 0
        self.world_size = 1
        self.initialized = False

    def init_process_group(self, backend: str = "nccl", init_method: str = "env://", timeout_s: float = 120.0,
                           device_id: Optional[torch.device] = None):
        if not dist.is_initialized():
            kw = dict(backend=backend, init_method=init_method, timeout=timedelta(seconds=timeout_s))
            if device_id is not None:
                kw["device_id"] = device_id
            dist.init_process_group(**kw)
        return self.attach()

    def attach(self, group: Optional[dist.ProcessGroup] = None):
        """Use an existing process group (default: the world, or its first ``ep_size`` ranks
        when the world is larger -- every rank of the world must then call this, as
        ``dist.new_group`` requires).  ``rank`` and ``world_size`` are this process's rank and
        the size *within* the group; a process outside the group gets rank -1."""
        if group is None:
            ws = dist.get_world_size()
            if ws < self.ep_size:
                raise ValueError(f"world size {ws} < EP size {self.ep_size}")
            if self.ep_size != ws:
                group = dist.new_group(list(range(self.ep_size)))
        self.world_size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world_size != self.ep_size:
            raise ValueError(f"process group of {self.world_size} ranks for EP size {self.ep_size}")
        self.group = group
        self.initialized = True
        return self

    def all_to_all(self, output_tensor, input_tensor, output_split_sizes=None, input_split_sizes=None):
        dist.all_to_all_single(output_tensor, input_tensor, output_split_sizes, input_split_sizes, group=self.group)
        return output_tensor

    def all_to_all_async(self, output_tensor, input_tensor, output_split_sizes=None, input_split_sizes=None):
        """Enqueue an all-to-all-v and return its work handle; ``wait()`` on it orders the
        caller's current CUDA stream after the transfer without blocking the host."""
        return dist.all_to_all_single(output_tensor, input_tensor, output_split_sizes, input_split_sizes,
                                      group=self.group, async_op=True)

    def all_reduce(self, tensor):
        dist.all_reduce(tensor, group=self.group)
        return tensor


# largest rows-per-expert bound for which the grouped GEMM entry point picks the decode kernels
DECODE_MAX_ROWS = 64


class CudaExpertBackend:
    """Local expert compute on the sm_100a library (the product path)."""

    def __init__(self, local: W4A16Experts, top_k: int):
        self.ex = local
        self.top_k = top_k
        self.num_local = local.num_experts      # routed experts on this rank
        self.num_shared = local.num_shared
        # when a list, every gate/up GEMM appends (start event, end event, rows) on the current
        # stream (used to time the per-rank kernel inside an expert-parallel step)
        self.gemm_timer = None
        # CTAs of the persistent GEMMs (None: one per SM); fewer leave SMs to the all-to-all
        # kernels of other micro-batches running beside the GEMMs
        self.sm_limit = None

    def route(self, x, gate_weight, gate_bias):
        ids, w, counts, offsets, sidx, pos = ops.fused_gate_topk_ex(x, gate_weight, self.top_k, gate_bias)[:6]
        return ids, w, counts, offsets, sidx, pos

    def gather(self, x, sorted_idx):
        from . import capi
        rows = torch.empty(sorted_idx.numel(), x.shape[1], dtype=x.dtype, device=x.device)
        capi.call("lmoe_permute_rows", x.data_ptr(), x.element_size(), sorted_idx.data_ptr(), sorted_idx.numel(),
                  x.shape[1],
                  self.top_k, rows.data_ptr(), capi.stream_handle())
        return rows

    def take(self, rows, index):
        """rows[index] (int32 index on the device) with the library's row gather."""
        from . import capi
        out = torch.empty(index.numel(), rows.shape[1], dtype=rows.dtype, device=rows.device)
        capi.call("lmoe_permute_rows", rows.data_ptr(), rows.element_size(), index.data_ptr(), index.numel(),
                  rows.shape[1], 1, out.data_ptr(), capi.stream_handle())
        return out

    def capacity_send_plan(self, counts, sidx, pos, T, k, ep, epr, C):
        from . import capi
        send_index = torch.empty(ep * C, dtype=torch.int32, device=counts.device)
        combine_pos = torch.empty(T * k, dtype=torch.int32, device=counts.device)
        capi.call("lmoe_capacity_send_plan", counts.data_ptr(), sidx.data_ptr(), pos.data_ptr(), T, k, ep, epr, C,
                  send_index.data_ptr(), combine_pos.data_ptr(), capi.stream_handle())
        return send_index, combine_pos

    def capacity_receive_plan(self, recv_counts, ep, epr, C, S, T):
        from . import capi
        dev = recv_counts.device
        regroup = torch.empty(ep * C, dtype=torch.int32, device=dev)
        restore = torch.empty(ep * C, dtype=torch.int32, device=dev)
        seg_offsets = torch.empty(epr + S + 2, dtype=torch.int32, device=dev)
        capi.call("lmoe_capacity_receive_plan", recv_counts.data_ptr(), ep, epr, C, S, T, regroup.data_ptr(),
                  restore.data_ptr(), seg_offsets.data_ptr(), capi.stream_handle())
        return regroup, restore, seg_offsets

    def experts(self, rows, seg_offsets, seg_expert, num_seg, max_rows, down_max_rows=None):
        """Both projections of the segments.  max_rows / down_max_rows: the rows-per-segment
        hints of the gate/up and down GEMMs (<= 64 selects the decode kernels)."""
        if self.sm_limit is None:
            return self._experts(rows, seg_offsets, seg_expert, num_seg, max_rows, down_max_rows)
        from . import capi
        prev = capi.lib().lmoe_get_gemm_sm_limit()
        capi.call("lmoe_set_gemm_sm_limit", int(self.sm_limit))
        try:
            return self._experts(rows, seg_offsets, seg_expert, num_seg, max_rows, down_max_rows)
        finally:
            capi.call("lmoe_set_gemm_sm_limit", prev)

    def _experts(self, rows, seg_offsets, seg_expert, num_seg, max_rows, down_max_rows=None):
        e = self.ex
        h = self.gate_up(rows, seg_offsets, seg_expert, num_seg, max_rows)
        return ops.w4a16_grouped_gemm(h, e.w2_packed, seg_offsets, num_seg, e.hidden_size, e.group_size, 0,
                                      None, None, 0, max_rows if down_max_rows is None else down_max_rows,
                                      seg_expert)

    def gate_up(self, rows, seg_offsets, seg_expert, num_seg, max_rows):
        """The gate/up projection with the SwiGLU epilogue (h), timed when gemm_timer is set."""
        e = self.ex
        if self.gemm_timer is not None:
            ev0 = torch.cuda.Event(enable_timing=True)
            ev0.record()
        h = ops.w4a16_grouped_gemm(rows, e.w13_packed, seg_offsets, num_seg, 2 * e.ffn_size, e.group_size, 1,
                                   None, None, 0, max_rows, seg_expert)
        if self.gemm_timer is not None:
            ev1 = torch.cuda.Event(enable_timing=True)
            ev1.record()
            # rows the GEMM computed: every segment but the holes (weight matrix -1); read
            # after the end event, so the copy is outside the timed launch
            n = seg_offsets[1: num_seg + 1].long() - seg_offsets[:num_seg].long()
            self.gemm_timer.append((ev0, ev1, int((n * (seg_expert[:num_seg] >= 0)).sum().item())))
        return h

    def combine(self, rows, positions, weights, T, extra, num_extra):
        return ops.combine_rows(rows, positions, weights, T, self.top_k, extra, num_extra)

    def make_exchange(self, group, config, capacity_tokens):
        """The peer-memory exchange (symmetric buffers mapped over CUDA IPC; collective)."""
        from .peer_exchange import PeerExchange
        return PeerExchange(group, config.num_experts, capacity_tokens, config.top_k, config.num_shared,
                            config.hidden_size, torch.device("cuda", torch.cuda.current_device()))

    def down_to_peers(self, px, h, seg_expert, num_seg, num_tokens):
        """The down projection whose epilogue returns every routed row to its source's slot."""
        e = self.ex
        px.down_gemm(h, e.w2_packed, e.ffn_size, e.group_size, seg_expert, num_seg, self.num_local + self.num_shared,
                     num_tokens)


class ExpertParallelW4A16Layer(HostBufferCalls, torch.nn.Module):
    """Expert-parallel W4A16 MoE layer: experts sharded by contiguous blocks over ep ranks.
    forward_host / forward_host_async (host-resident activations) run every call as one token
    range, so all ranks take the same steps."""

    _host_ranges = False

    def __init__(self, config: ExpertParallelConfig, ep_group: ExpertParallelGroup, gate_weight: torch.Tensor,
                 backend, gate_bias: Optional[torch.Tensor] = None, micro_batches: int = 1,
                 dispatch: str = "exact", capacity_tokens: Optional[int] = None, sm_reserve: Optional[int] = None):
        super().__init__()
        if dispatch not in ("exact", "capacity", "p2p"):
            raise ValueError(f"dispatch must be 'exact', 'capacity' or 'p2p', not {dispatch!r}")
        if dispatch in ("capacity", "p2p") and (capacity_tokens is None or int(capacity_tokens) < 1):
            raise ValueError(f"{dispatch} dispatch needs capacity_tokens >= 1 (the same on every rank)")
        self.dispatch = dispatch
        self.capacity_tokens = int(capacity_tokens) if capacity_tokens is not None else None
        self.config = config
        self.ep_group = ep_group
        self.gate_weight = gate_weight
        self.gate_bias = gate_bias
        self.backend = backend
        self.experts_per_rank = config.experts_per_rank
        self.local_expert_start = ep_group.rank * self.experts_per_rank
        self.local_expert_end = self.local_expert_start + self.experts_per_rank
        self.micro_batches = max(1, int(micro_batches))   # must be equal on all ranks
        # SMs left free by the GEMMs while micro-batches overlap (default 16 with more than
        # one micro-batch, 0 otherwise)
        self.sm_reserve = (16 if self.micro_batches > 1 else 0) if sm_reserve is None else int(sm_reserve)
        if self.sm_reserve > 0 and hasattr(backend, "sm_limit") and torch.cuda.is_available():
            props = torch.cuda.get_device_properties(torch.cuda.current_device())
            backend.sm_limit = max(1, props.multi_processor_count - self.sm_reserve)
        # kernels of ours per forward: router, gather, gate/up GEMM, down GEMM, combine per
        # micro-batch (set by the last forward)
        self.kernels_per_step = 5
        self._seg_cache = {}
        # dispatch="p2p": rows move through peer memory (collective setup of the symmetric
        # buffers here, outside any CUDA graph capture)
        self.exchange = None
        if dispatch == "p2p":
            if not hasattr(backend, "make_exchange"):
                raise ValueError("p2p dispatch needs a backend that provides the peer exchange")
            self.exchange = backend.make_exchange(ep_group, config, self.capacity_tokens)

    @classmethod
    def from_full(cls, gate_weight: torch.Tensor, experts: W4A16Experts, top_k: int,
                  group: Optional[dist.ProcessGroup] = None, gate_bias: Optional[torch.Tensor] = None,
                  micro_batches: int = 1, dispatch: str = "exact", capacity_tokens: Optional[int] = None,
                  sm_reserve: Optional[int] = None):
        """Build this rank's layer from the full (all-expert) prepacked weights."""
        ws = dist.get_world_size(group)
        g = ExpertParallelGroup(ws).attach(group)
        if g.rank < 0:
            raise ValueError("this process is not a member of the expert-parallel group")
        cfg = ExpertParallelConfig(num_experts=experts.num_experts, top_k=top_k, hidden_size=experts.hidden_size,
                                   intermediate_size=experts.ffn_size, ep_size=ws, group_size=experts.group_size,
                                   num_shared=experts.num_shared)
        local = slice_experts(experts, g.rank * cfg.experts_per_rank, (g.rank + 1) * cfg.experts_per_rank)
        return cls(cfg, g, gate_weight.to(torch.bfloat16).contiguous(), CudaExpertBackend(local, top_k), gate_bias,
                   micro_batches, dispatch, capacity_tokens, sm_reserve)

    def _segments(self, device):
        key = (str(device),)
        if key not in self._seg_cache:
            ep, epr, S = self.ep_group.ep_size, self.experts_per_rank, self.config.num_shared
            seg = [i % epr for i in range(ep * epr)] + [epr + s for s in range(S)]
            self._seg_cache[key] = torch.tensor(seg, dtype=torch.int32, device=device)
        return self._seg_cache[key]

    def _gemm_hints(self):
        """Rows-per-segment hints of the gate/up and down GEMMs of a capacity-bounded step,
        from the expected rows per local expert (ep * Tc * k / E; the segments' real sizes
        stay on the device).  Measured on one Mixtral expert (gate/up 28672 x 4096, down 4096 x
        14336) as a single segment: the decode kernel
        (32-row token blocks, the weights streamed once per block) wins the gate/up GEMM up
        to ~32 rows (39 against 50 us) and loses from 64 (68 against 52; 113 against 56 at
        128); its down GEMM wins up to 128 rows (55 against 82 us) and loses from ~192."""
        cfg = self.config
        est = self.ep_group.ep_size * self.capacity_tokens * cfg.top_k // cfg.num_experts
        big = max(est, DECODE_MAX_ROWS + 1)
        gu = DECODE_MAX_ROWS if est < DECODE_MAX_ROWS else big
        dn = DECODE_MAX_ROWS if est <= 2 * DECODE_MAX_ROWS else big
        return gu, dn

    def _capacity_segments(self, device):
        key = ("cap", str(device))
        if key not in self._seg_cache:
            epr, S = self.experts_per_rank, self.config.num_shared
            seg = list(range(epr)) + [-1] + [epr + s for s in range(S)]
            self._seg_cache[key] = torch.tensor(seg, dtype=torch.int32, device=device)
        return self._seg_cache[key]

    def _forward_capacity(self, x: torch.Tensor) -> torch.Tensor:
        T, d = x.shape
        cfg, g, be = self.config, self.ep_group, self.backend
        ep, epr, k, S = g.ep_size, self.experts_per_rank, cfg.top_k, cfg.num_shared
        if T > self.capacity_tokens:
            raise ValueError(f"{T} tokens exceed capacity_tokens={self.capacity_tokens}")
        C = self.capacity_tokens * k                  # rows per destination block
        dev = x.device
        self.kernels_per_step = 9
        if T > 0:
            ids, w, counts, offsets, sidx, pos = be.route(x, self.gate_weight, self.gate_bias)
            counts = counts.view(ep, epr).to(torch.int32)
            send_index, combine_pos = be.capacity_send_plan(counts, sidx, pos, T, k, ep, epr, C)
            send = be.gather(x, send_index)
        else:
            counts = torch.zeros(ep, epr, dtype=torch.int32, device=dev)
            send = torch.zeros(ep * C, d, dtype=x.dtype, device=dev)
        # the counts travel in an all-to-all; only the device reads them
        recv_counts = torch.empty(ep, epr, dtype=torch.int32, device=dev)
        g.all_to_all(recv_counts, counts.contiguous())
        recv = torch.empty(ep * C, d, dtype=x.dtype, device=dev)
        g.all_to_all(recv, send)
        # regroup the received rows expert-major (each local expert one segment, so its weights
        # stream once whatever the number of source ranks); every source's padding becomes one
        # trailing hole
        regroup, restore, seg_offsets = be.capacity_receive_plan(recv_counts, ep, epr, C, S, T)
        rows_em = torch.empty(ep * C + S * T, d, dtype=x.dtype, device=dev)
        rows_em[: ep * C] = be.take(recv, regroup)
        for s in range(S):
            rows_em[ep * C + s * T: ep * C + (s + 1) * T].copy_(x)
        out_em = be.experts(rows_em, seg_offsets, self._capacity_segments(dev), epr + 1 + S, *self._gemm_hints())
        out = be.take(out_em, restore)                                              # back to capacity order
        ret = torch.empty(ep * C, d, dtype=x.dtype, device=dev)
        g.all_to_all(ret, out)
        extra = out_em[ep * C:] if S else None
        if T == 0:
            return torch.empty(0, d, dtype=x.dtype, device=dev)
        return be.combine(ret, combine_pos, w, T, extra, S)

    def _forward_p2p(self, x: torch.Tensor) -> torch.Tensor:
        """Dispatch and return through peer memory: counts exchange, fused permute + send,
        the local grouped GEMMs on the rows region, fused send-back, weighted combine."""
        T, d = x.shape
        cfg, be, px = self.config, self.backend, self.exchange
        epr, k, S = self.experts_per_rank, cfg.top_k, cfg.num_shared
        if T > self.capacity_tokens:
            raise ValueError(f"{T} tokens exceed capacity_tokens={self.capacity_tokens}")
        dev = x.device
        self.kernels_per_step = 8
        x = x.contiguous()
        if T > 0:
            ids, w, counts, offsets, sidx, pos = be.route(x, self.gate_weight, self.gate_bias)
        else:
            counts = torch.zeros(cfg.num_experts, dtype=torch.int32, device=dev)
            ids = w = offsets = sidx = None
        px.exchange_counts(counts, T)
        px.dispatch(x, sidx, ids, offsets)
        px.wait_rows(T)
        segs, nseg = self._capacity_segments(dev), epr + 1 + S
        gu_hint, dn_hint = self._gemm_hints()
        if dn_hint > DECODE_MAX_ROWS:
            # large segments: the down GEMM's epilogue writes the routed rows straight into
            # their sources' ret slots (the return transfer overlaps the GEMM's tiles)
            h = be.gate_up(px.rows, px.seg_offsets, segs, nseg, gu_hint)
            be.down_to_peers(px, h, segs, nseg, T)
            shared = px.shared_out
        else:
            # decode-sized down GEMM (writes locally), then one copy kernel sends the rows back
            out = be.experts(px.rows, px.seg_offsets, segs, nseg, gu_hint, dn_hint)
            px.send_back(out, T)
            shared = out[px.routed_rows:]
        px.wait_returns(T)
        if T == 0:
            return torch.empty(0, d, dtype=x.dtype, device=dev)
        key = ("slots", T * k, str(dev))
        if key not in self._seg_cache:
            self._seg_cache[key] = torch.arange(T * k, dtype=torch.int32, device=dev)
        extra = shared[: S * T] if S else None
        return be.combine(px.ret[: T * k], self._seg_cache[key], w, T, extra, S)

    def close(self):
        """Release the peer-exchange buffers (collective; p2p dispatch only)."""
        if self.exchange is not None:
            self.exchange.close()
            self.exchange = None

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        x = hidden_states.reshape(-1, hidden_states.shape[-1])
        if self.dispatch == "capacity":
            return self._forward_capacity(x).view(hidden_states.shape)
        if self.dispatch == "p2p":
            return self._forward_p2p(x).view(hidden_states.shape)
        T, d = x.shape
        cfg, g, be = self.config, self.ep_group, self.backend
        ep, epr, k, S = g.ep_size, self.experts_per_rank, cfg.top_k, cfg.num_shared
        dev = x.device
        nmb = self.micro_batches
        bounds = [(T * m // nmb, T * (m + 1) // nmb) for m in range(nmb)]
        self.kernels_per_step = 5 * nmb

        # 1-2. route and gather every micro-batch (destination-rank order)
        mbs = []
        for a, b in bounds:
            xm = x[a:b]
            ids, w, counts, offsets, sidx, pos = be.route(xm, self.gate_weight, self.gate_bias)
            mbs.append({"x": xm, "T": b - a, "w": w, "pos": pos, "counts": counts, "rows": be.gather(xm, sidx)})

        # 3. one count exchange for all micro-batches: send[r, m, e] = rows of micro-batch m
        #    for expert e of rank r; recv[s, m, e] = rows rank s sends us; one host copy
        send_counts = torch.stack([mb["counts"].view(ep, epr) for mb in mbs], 1).contiguous()
        recv_counts = torch.empty_like(send_counts)
        g.all_to_all(recv_counts, send_counts)
        both = torch.cat([send_counts.flatten(), recv_counts.flatten()]).cpu()
        send_h = both[: ep * nmb * epr].view(ep, nmb, epr)
        recv_h = both[ep * nmb * epr:].view(ep, nmb, epr)

        # 4. dispatch all micro-batches; NCCL runs them in order on its own stream
        for m, mb in enumerate(mbs):
            mb["send_splits"] = send_h[:, m].sum(1).tolist()
            mb["recv_h"] = recv_h[:, m]
            mb["recv_splits"] = mb["recv_h"].sum(1).tolist()
            R = int(sum(mb["recv_splits"]))
            mb["R"] = R
            mb["recv"] = torch.empty(R + S * mb["T"], d, dtype=x.dtype, device=dev)
            mb["work"] = g.all_to_all_async(mb["recv"][:R], mb["rows"], mb["recv_splits"], mb["send_splits"])

        # 5-6. GEMMs of micro-batch m once its rows are here; its combine all-to-all then
        #      overlaps the GEMMs of the next micro-batch
        for mb in mbs:
            mb["work"].wait()
            R, Tm, recv = mb["R"], mb["T"], mb["recv"]
            for s in range(S):                                       # shared experts: local tokens
                recv[R + s * Tm: R + (s + 1) * Tm].copy_(mb["x"])
            seg_counts = mb["recv_h"].flatten().tolist() + [Tm] * S
            offs = [0]
            for c in seg_counts:
                offs.append(offs[-1] + int(c))
            seg_offsets = torch.tensor(offs, dtype=torch.int32).to(dev, non_blocking=True)
            max_rows = max(seg_counts) if seg_counts else 0
            out = be.experts(recv, seg_offsets, self._segments(dev), len(seg_counts), max_rows)
            mb["out"] = out
            mb["ret"] = torch.empty(Tm * k, d, dtype=x.dtype, device=dev)
            mb["work"] = g.all_to_all_async(mb["ret"], out[:R].contiguous(), mb["send_splits"], mb["recv_splits"])

        # 7. weighted combine of each micro-batch
        ys = []
        for mb in mbs:
            mb["work"].wait()
            extra = mb["out"][mb["R"]:] if S else None
            ys.append(be.combine(mb["ret"], mb["pos"], mb["w"], mb["T"], extra, S))
        y = ys[0] if nmb == 1 else torch.cat(ys)
        return y.view(hidden_states.shape)


def capacity_send_plan_torch(counts, sidx, pos, T: int, k: int, ep: int, epr: int, C: int):
    """The fixed-capacity send plan (lmoe_capacity_send_plan) in torch index operations:
    (send_index [ep * C], combine_pos [T * k]), int32 on counts' device."""
    dev = counts.device
    cnt_r = counts.view(ep, epr).to(torch.int64).sum(1)
    end_r = torch.cumsum(cnt_r, 0)
    start_r = end_r - cnt_r
    j = torch.arange(T * k, device=dev, dtype=torch.int64)
    r_of_j = torch.searchsorted(end_r, j, right=True)
    p = r_of_j * C + (j - start_r[r_of_j])          # sorted row -> slot of its destination's block
    c = torch.arange(C, device=dev, dtype=torch.int64)
    src = (start_r[:, None] + c[None, :]).clamp(max=max(T * k - 1, 0))
    send_index = torch.where(c[None, :] < cnt_r[:, None], sidx.long()[src], torch.zeros_like(src))
    return send_index.to(torch.int32).flatten(), p[pos.long()].to(torch.int32)


def capacity_receive_plan_torch(recv_counts, ep: int, epr: int, C: int, S: int, T: int):
    """The fixed-capacity receive plan (lmoe_capacity_receive_plan) in torch index operations:
    (regroup [ep * C], restore [ep * C], seg_offsets [epr + S + 2]), int32."""
    dev = recv_counts.device
    rc = recv_counts.view(ep, epr).long()
    cnt = torch.cat([rc, C - rc.sum(1, keepdim=True)], 1)                        # [ep, epr + 1]
    src_start = (torch.arange(ep, device=dev) * C)[:, None] + torch.cumsum(cnt, 1) - cnt
    cnt_em = cnt.t().contiguous().flatten()                                       # (expert, source)
    dst_start = torch.cumsum(cnt_em, 0) - cnt_em
    jj = torch.arange(ep * C, device=dev)
    kk = torch.searchsorted(dst_start, jj, right=True) - 1
    regroup = src_start.t().contiguous().flatten()[kk] + (jj - dst_start[kk])
    restore = torch.empty_like(regroup)
    restore[regroup] = jj
    seg_counts = cnt_em.view(epr + 1, ep).sum(1)
    if S:
        seg_counts = torch.cat([seg_counts, torch.full((S,), T, dtype=torch.long, device=dev)])
    seg_offsets = torch.cat([torch.zeros(1, dtype=torch.long, device=dev), torch.cumsum(seg_counts, 0)])
    return regroup.to(torch.int32), restore.to(torch.int32), seg_offsets.to(torch.int32)


def slice_experts(ex: W4A16Experts, e0: int, e1: int) -> W4A16Experts:
    """Routed experts [e0, e1) plus every shared expert, from full prepacked weights.

    The prepacked layouts are expert-major, so an expert range is one contiguous slice.
    """
    if not 0 <= e0 <= e1 <= ex.num_experts:
        raise ValueError(f"expert range [{e0}, {e1}) outside the {ex.num_experts} routed experts")
    Et = ex.num_experts + ex.num_shared

    def part(t, idx):
        per = t.numel() // Et
        return torch.cat([t[i * per:(i + 1) * per] for i in idx]) if idx else t[:0]

    idx = list(range(e0, e1)) + list(range(ex.num_experts, Et))
    return W4A16Experts(part(ex.w13_packed, idx), part(ex.w2_packed, idx), e1 - e0, ex.num_shared,
                        ex.hidden_size, ex.ffn_size, ex.group_size, None)


def init_distributed(backend: str = "nccl", timeout_s: float = 120.0):
    """Rendezvous from the torchrun environment (comm_group.py:104-138 of the reference)."""
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1 and not dist.is_initialized():
        kw = dict(backend=backend, timeout=timedelta(seconds=timeout_s))
        if backend == "nccl":
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(**kw)
    return ws, rank
