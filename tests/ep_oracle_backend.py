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

    def experts(self, rows, seg_offsets, seg_expert, num_seg, max_rows, down_max_rows=None):
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

    # --- peer-memory exchange (dispatch="p2p"), restated on CPU ranks -----------------
    def make_exchange(self, group, config, capacity_tokens):
        return EmulatedPeerExchange(group, config.num_experts, capacity_tokens, config.top_k, config.num_shared,
                                    config.hidden_size)

    def gate_up(self, rows, seg_offsets, seg_expert, num_seg, max_rows):
        return rows   # the whole expert MLP runs in down_to_peers

    def down_to_peers(self, px, h, seg_expert, num_seg, num_tokens):
        out = self.experts(h, px.seg_offsets, seg_expert, num_seg, None)
        px.send_back(out, num_tokens)
        S, T = self.num_shared, num_tokens
        if S:
            px.shared_out[: S * T] = out[px.routed_rows: px.routed_rows + S * T]


class EmulatedPeerExchange:
    """The peer-memory exchange of light_moe_b200/csrc/ep_p2p.cu restated for CPU ranks: the
    same buffer regions (rows expert-major by source, meta words, returned slots, shared
    rows), the same count-matrix arithmetic for segment offsets and destination positions,
    with gloo all-to-alls standing in for the peer stores.  Test infrastructure only."""

    def __init__(self, group, num_experts, capacity_tokens, top_k, num_shared, hidden):
        import torch.distributed as dist
        self.dist = dist
        self.pg = group.group
        self.ep, self.me = group.ep_size, group.rank
        self.E, self.Tc, self.k, self.S, self.d = num_experts, int(capacity_tokens), top_k, num_shared, hidden
        self.epr = num_experts // self.ep
        self.routed_rows = self.ep * self.Tc * top_k
        self.rows = torch.zeros(self.routed_rows + num_shared * self.Tc, hidden)
        self.meta = torch.zeros(self.routed_rows + num_shared * self.Tc, dtype=torch.int64)
        self.meta[self.routed_rows:] = (self.ep << 24) + torch.arange(num_shared * self.Tc)
        self.ret = torch.zeros(self.Tc * top_k, hidden)
        self.shared_out = torch.zeros(max(num_shared * self.Tc, 1), hidden)
        self.seg_offsets = torch.zeros(self.epr + 2 + num_shared, dtype=torch.int32)
        self.dst_base = torch.zeros(num_experts, dtype=torch.int64)

    def exchange_counts(self, counts, num_tokens):
        ep, E, epr, me = self.ep, self.E, self.epr, self.me
        mine = counts.to(torch.int64).reshape(E)
        allc = [torch.empty_like(mine) for _ in range(ep)]
        self.dist.all_gather(allc, mine, group=self.pg)
        cnt = torch.stack(allc)                                   # [source, expert]
        per_expert = cnt.sum(0)
        seg = [0]
        for l in range(epr):
            seg.append(seg[-1] + int(per_expert[me * epr + l]))
        seg.append(self.routed_rows)
        seg += [self.routed_rows + (s + 1) * num_tokens for s in range(self.S)]
        self.seg_offsets = torch.tensor(seg, dtype=torch.int32)
        for e in range(E):
            r = e // epr
            self.dst_base[e] = int(per_expert[r * epr: e].sum()) + int(cnt[:me, e].sum())

    def _exchange(self, dest_rank, payload_rows, payload_idx):
        """Send payload rows / indices to their destination ranks; returns what arrived."""
        order = torch.argsort(dest_rank, stable=True)
        send_n = torch.bincount(dest_rank, minlength=self.ep)
        recv_n = torch.empty_like(send_n)
        self.dist.all_to_all_single(recv_n, send_n, group=self.pg)
        rows_in = torch.empty(int(recv_n.sum()), self.d)
        idx_in = torch.empty(int(recv_n.sum()), payload_idx.shape[1], dtype=torch.int64)
        self.dist.all_to_all_single(rows_in, payload_rows[order].contiguous(), recv_n.tolist(), send_n.tolist(),
                                    group=self.pg)
        self.dist.all_to_all_single(idx_in, payload_idx[order].contiguous(), recv_n.tolist(), send_n.tolist(),
                                    group=self.pg)
        return rows_in, idx_in

    def dispatch(self, x, sorted_idx, ids, offsets):
        T, k = x.shape[0], self.k
        if T:
            f = sorted_idx.long()
            e = ids.reshape(-1).long()[f]
            pos = self.dst_base[e] + (torch.arange(T * k) - offsets.long()[e])
            meta = (self.me << 24) + f
            rows_in, idx_in = self._exchange(e // self.epr, x[f // k], torch.stack([pos, meta], 1))
        else:
            rows_in, idx_in = self._exchange(torch.zeros(0, dtype=torch.int64), torch.zeros(0, self.d),
                                             torch.zeros(0, 2, dtype=torch.int64))
        self.rows[idx_in[:, 0]] = rows_in
        self.meta[idx_in[:, 0]] = idx_in[:, 1]
        for s in range(self.S):
            self.rows[self.routed_rows + s * T: self.routed_rows + (s + 1) * T] = x

    def wait_rows(self, num_tokens):
        pass

    def send_back(self, out, num_tokens):
        R = int(self.seg_offsets[self.epr])
        m = self.meta[:R]
        rows_in, idx_in = self._exchange(m >> 24, out[:R], (m & 0xFFFFFF)[:, None])
        self.ret[idx_in[:, 0]] = rows_in

    def wait_returns(self, num_tokens):
        pass

    def error(self):
        return 0

    def close(self):
        pass
