"""CPU expert backend for the expert-parallel tests (test infrastructure: uses the oracle).

Implements the backend interface of light_moe_b200.expert_parallel with the CPU oracle so
the multi-rank bookkeeping (count exchange, split sizes, segment offsets, segment -> expert
map, order restoration) runs on gloo CPU ranks.
"""
import numpy as np
import torch

import oracle


class OracleExpertBackend:
    def __init__(self, w1, w3, w2, top_k, num_shared=0):
        # w*: fp32 numpy, local routed experts followed by the shared ones
        self.w1, self.w3, self.w2 = w1, w3, w2
        self.top_k = top_k
        self.num_shared = num_shared

    def route(self, x, gate_weight, gate_bias):
        lg = x.numpy().astype(np.float32) @ gate_weight.numpy().astype(np.float32).T
        if gate_bias is not None:
            lg = lg + gate_bias.numpy()[None, :]
        ids, w = oracle.route(lg.astype(np.float32), self.top_k)
        counts, offsets, sidx = oracle.counts_offsets(ids, gate_weight.shape[0])
        pos = np.empty_like(sidx)
        pos[sidx] = np.arange(sidx.size, dtype=np.int32)
        t = torch.from_numpy
        return t(ids), t(w), t(counts), t(offsets), t(sidx), t(pos)

    def gather(self, x, sorted_idx):
        return x[(sorted_idx // self.top_k).long()].contiguous()

    def capacity_send_plan(self, counts, sidx, pos, T, k, ep, epr, C):
        from light_moe_b200.expert_parallel import capacity_send_plan_torch
        return capacity_send_plan_torch(counts, sidx, pos, T, k, ep, epr, C)

    def capacity_receive_plan(self, recv_counts, ep, epr, C, S, T):
        from light_moe_b200.expert_parallel import capacity_receive_plan_torch
        return capacity_receive_plan_torch(recv_counts, ep, epr, C, S, T)

    def take(self, rows, index):
        return rows[index.long()].contiguous()

    def experts(self, rows, seg_offsets, seg_expert, num_seg, max_rows):
        out = torch.zeros(rows.shape[0], self.w2.shape[1], dtype=rows.dtype)
        off = seg_offsets.tolist()
        se = seg_expert.tolist()
        for i in range(num_seg):
            a, b = off[i], off[i + 1]
            if b > a and se[i] != -1:   # -1: a hole (padding rows), skipped like the GEMMs do
                e = se[i]
                y = oracle.expert_mlp_ref(rows[a:b].numpy(), self.w1[e], self.w3[e], self.w2[e])
                out[a:b] = torch.from_numpy(y)
        return out

    def combine(self, rows, positions, weights, T, extra, num_extra):
        k = self.top_k
        y = torch.zeros(T, rows.shape[1], dtype=rows.dtype)
        for j in range(k):
            y += rows[positions.view(T, k)[:, j].long()] * weights.view(T, k)[:, j:j + 1]
        for s in range(num_extra):
            y += extra[s * T:(s + 1) * T]
        return y
