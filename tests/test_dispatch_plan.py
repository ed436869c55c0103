"""Index plans of the fixed-capacity expert-parallel exchange.

CPU: the torch statement of the plans (used by the CPU expert backends) against plain loops.
GPU: the plan kernels (lmoe_capacity_send_plan / lmoe_capacity_receive_plan) against the torch
statement, bit for bit, on random counts -- full blocks, empty ranks, shared segments."""
import pytest
import torch

from light_moe_b200.expert_parallel import capacity_receive_plan_torch, capacity_send_plan_torch


def _case(ep, epr, T, k, C, seed, full_rank=None):
    gen = torch.Generator().manual_seed(seed)
    n = T * k
    # counts per (destination rank, expert) summing to n; one rank may take all rows
    if full_rank is not None:
        counts = torch.zeros(ep, epr, dtype=torch.int32)
        counts[full_rank] = torch.bincount(torch.randint(0, epr, (n,), generator=gen), minlength=epr).to(torch.int32)
    else:
        counts = torch.bincount(torch.randint(0, ep * epr, (n,), generator=gen), minlength=ep * epr)
        counts = counts.view(ep, epr).to(torch.int32)
    sidx = torch.randperm(n, generator=gen).to(torch.int32)      # sorted row -> (token, choice)
    pos = torch.empty(n, dtype=torch.int32)
    pos[sidx.long()] = torch.arange(n, dtype=torch.int32)        # (token, choice) -> sorted row
    return counts, sidx, pos


def _recv_counts(ep, epr, C, seed):
    gen = torch.Generator().manual_seed(seed)
    rc = torch.zeros(ep, epr, dtype=torch.int32)
    for s in range(ep):
        n = int(torch.randint(0, C + 1, (1,), generator=gen))
        rc[s] = torch.bincount(torch.randint(0, epr, (n,), generator=gen), minlength=epr).to(torch.int32)
    return rc


def _send_loops(counts, sidx, pos, T, k, ep, epr, C):
    send = [0] * (ep * C)
    start, acc = [], 0
    for r in range(ep):
        start.append(acc)
        n_r = int(counts[r].sum())
        for c in range(n_r):
            send[r * C + c] = int(sidx[acc + c])
        acc += n_r
    comb = []
    for j in range(T * k):
        sr = int(pos[j])
        r = max(i for i in range(ep) if start[i] <= sr)
        comb.append(r * C + sr - start[r])
    return send, comb


def _receive_loops(rc, ep, epr, C, S, T):
    regroup, seg = [], [0]
    for e in range(epr + 1):
        for s in range(ep):
            used = int(rc[s, :e].sum())
            n = int(rc[s, e]) if e < epr else C - int(rc[s].sum())
            regroup += [s * C + used + i for i in range(n)]
        seg.append(len(regroup))
    seg += [len(regroup) + (i + 1) * T for i in range(S)]
    restore = [0] * len(regroup)
    for p, q in enumerate(regroup):
        restore[q] = p
    return regroup, restore, seg


PLAN_CASES = [(1, 8, 64, 2, 128, 0, None), (2, 4, 64, 2, 128, 0, None), (4, 2, 33, 4, 160, 2, None),
              (8, 1, 7, 2, 14, 1, 3), (8, 8, 64, 2, 128, 0, None), (3, 5, 1, 3, 3, 0, 0)]


@pytest.mark.parametrize("ep,epr,T,k,C,S,full", PLAN_CASES)
def test_plan_torch_matches_loops(ep, epr, T, k, C, S, full):
    counts, sidx, pos = _case(ep, epr, T, k, C, seed=ep * 100 + epr, full_rank=full)
    send, comb = capacity_send_plan_torch(counts, sidx, pos, T, k, ep, epr, C)
    send_l, comb_l = _send_loops(counts, sidx, pos, T, k, ep, epr, C)
    assert send.tolist() == send_l and comb.tolist() == comb_l
    rc = _recv_counts(ep, epr, C, seed=ep + epr)
    regroup, restore, seg = capacity_receive_plan_torch(rc, ep, epr, C, S, T)
    rg_l, rs_l, seg_l = _receive_loops(rc, ep, epr, C, S, T)
    assert regroup.tolist() == rg_l and restore.tolist() == rs_l and seg.tolist() == seg_l


@pytest.mark.gpu
@pytest.mark.parametrize("ep,epr,T,k,C,S,full", PLAN_CASES + [(16, 8, 128, 8, 1024, 1, None),
                                                             (64, 4, 256, 8, 2048, 2, 63)])
def test_plan_kernels_match_torch(ep, epr, T, k, C, S, full):
    from light_moe_b200.expert_parallel import CudaExpertBackend
    dev = torch.device("cuda", 0)
    counts, sidx, pos = _case(ep, epr, T, k, C, seed=ep * 100 + epr, full_rank=full)
    counts, sidx, pos = counts.to(dev), sidx.to(dev), pos.to(dev)
    send, comb = CudaExpertBackend.capacity_send_plan(None, counts, sidx, pos, T, k, ep, epr, C)
    send_t, comb_t = capacity_send_plan_torch(counts, sidx, pos, T, k, ep, epr, C)
    rc = _recv_counts(ep, epr, C, seed=ep + epr).to(dev)
    plan = CudaExpertBackend.capacity_receive_plan(None, rc, ep, epr, C, S, T)
    plan_t = capacity_receive_plan_torch(rc, ep, epr, C, S, T)
    torch.cuda.synchronize()
    assert torch.equal(send, send_t) and torch.equal(comb, comb_t)
    for a, b in zip(plan, plan_t):
        assert torch.equal(a, b)


@pytest.mark.parametrize("ep,Tc,E,k,expect", [
    (1, 64, 8, 2, (64, 64)),        # 16 rows per expert: decode kernels for both GEMMs
    (2, 64, 8, 2, (64, 64)),        # 32 rows
    (4, 64, 8, 2, (65, 64)),        # 64 rows: prefill tiles for gate/up, decode down
    (8, 64, 8, 2, (128, 64)),       # 128 rows: still the decode down GEMM
    (8, 96, 8, 2, (192, 192)),      # 192 rows: prefill tiles for both (down fused with the return)
    (2, 8192, 8, 2, (4096, 4096)),  # prefill step
    (4, 9, 64, 6, (64, 64)),        # fine-grained decode: 3 rows per expert
])
def test_gemm_kernel_choice_follows_expected_rows_per_expert(ep, Tc, E, k, expect):
    from types import SimpleNamespace
    from light_moe_b200.expert_parallel import DECODE_MAX_ROWS, ExpertParallelW4A16Layer
    layer = SimpleNamespace(config=SimpleNamespace(top_k=k, num_experts=E), ep_group=SimpleNamespace(ep_size=ep),
                            capacity_tokens=Tc)
    gu, dn = ExpertParallelW4A16Layer._gemm_hints(layer)
    assert (gu, dn) == expect
    # a hint <= DECODE_MAX_ROWS selects the decode kernels in the grouped GEMM entry point
    assert (gu <= DECODE_MAX_ROWS) == (ep * Tc * k // E < DECODE_MAX_ROWS)
