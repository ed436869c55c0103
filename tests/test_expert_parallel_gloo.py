"""Expert-parallel layer on CPU ranks (gloo, world size 2 and 4).

The experts run on the CPU oracle backend; what is tested is the multi-rank logic of
ExpertParallelW4A16Layer -- count exchange, split sizes, segment offsets and the
segment -> expert map, dispatch / combine order, shared experts -- against the
single-process oracle layer on each rank's own tokens.  Also checks that a rank dying in
the middle of a step surfaces as an error on the surviving rank instead of a hang.
"""
import os
import socket
import sys
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights(E, S, d, F, g, seed=0):
    import oracle
    rng = np.random.default_rng(seed)
    dense = {n: (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.05))
             for n, shape in (("w1", (E + S, F, d)), ("w3", (E + S, F, d)), ("w2", (E + S, d, F)))}
    deq = {}
    for n, w in dense.items():
        q, s = oracle.quantize_w4(w, g)
        deq[n] = oracle.bf16_bits_to_f32(oracle.dequantize_w4(q, s, g))
    gw = (rng.standard_normal((E, d), dtype=np.float32) * np.float32(0.3)).astype(np.float32)
    return gw, deq


def _worker(rank, world, port, case, q):
    try:
        sys.path.insert(0, ROOT)
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        from datetime import timedelta
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
        import oracle
        from ep_oracle_backend import OracleExpertBackend
        from light_moe_b200.expert_parallel import (ExpertParallelConfig, ExpertParallelGroup,
                                                    ExpertParallelW4A16Layer)
        E, S, k, d, F, g, Ts = case["E"], case["S"], case["k"], case["d"], case["F"], case["g"], case["T"]
        gw, deq = _weights(E, S, d, F, g)
        if case.get("subgroups"):
            # two independent EP groups {0, 1} and {2, 3}: the layer must use its rank and size
            # within its own group, not in the world
            groups = [dist.new_group([0, 1]), dist.new_group([2, 3])]
            ep = 2
            grp = ExpertParallelGroup(ep).attach(groups[rank // 2])
        else:
            ep = world
            grp = ExpertParallelGroup(world).attach()
        epr = E // ep
        gr = grp.rank
        idx = list(range(gr * epr, (gr + 1) * epr)) + list(range(E, E + S))
        be = OracleExpertBackend(deq["w1"][idx], deq["w3"][idx], deq["w2"][idx], k, S)
        cfg = ExpertParallelConfig(num_experts=E, top_k=k, hidden_size=d, intermediate_size=F, ep_size=ep,
                                   group_size=g, num_shared=S)
        layer = ExpertParallelW4A16Layer(cfg, grp, torch.from_numpy(gw), be, micro_batches=case.get("mb", 1),
                                         dispatch=case.get("dispatch", "exact"), capacity_tokens=case.get("cap"))
        x = np.random.default_rng(100 + rank).standard_normal((Ts[rank], d), dtype=np.float32)
        if case.get("die") is not None and rank == case["die"]:
            be.route(torch.from_numpy(x), torch.from_numpy(gw), None)
            os._exit(3)   # leaves between steps, before the first collective of the step
        y = layer(torch.from_numpy(x)).numpy()
        shared = [(deq["w1"][E + s], deq["w3"][E + s], deq["w2"][E + s]) for s in range(S)] or None
        y_ref, _, _ = oracle.moe_layer_ref(x, gw, deq["w1"][:E], deq["w3"][:E], deq["w2"][:E], k, shared=shared)
        err = float(np.abs(y - y_ref).max() / max(np.abs(y_ref).max(), 1e-30)) if y.size else 0.0
        q.put((rank, "ok", err))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001 -- reported to the parent
        q.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc()}"))


def _run(world, case, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for p in procs:
        p.join(timeout)
        if p.is_alive():
            p.kill()
            p.join()
    while not q.empty():
        r, status, val = q.get()
        results[r] = (status, val)
    return results, [p.exitcode for p in procs]


@pytest.mark.parametrize("world,case", [
    (2, dict(E=8, S=0, k=2, d=64, F=64, g=64, T=[40, 40])),
    (2, dict(E=8, S=1, k=2, d=64, F=128, g=64, T=[5, 17])),
    (4, dict(E=8, S=0, k=3, d=64, F=64, g=64, T=[30, 1, 12, 25])),
    (2, dict(E=4, S=2, k=2, d=128, F=64, g=64, T=[3, 64])),
    # micro-batched dispatch / combine; rank 1 has fewer tokens than micro-batches
    (2, dict(E=8, S=1, k=2, d=64, F=128, g=64, T=[40, 1], mb=2)),
    (4, dict(E=8, S=0, k=3, d=64, F=64, g=64, T=[30, 2, 12, 25], mb=3)),
    # fine-grained routing shape: 64 experts (16 per rank), top-6, two shared experts
    (4, dict(E=64, S=2, k=6, d=64, F=64, g=64, T=[50, 9, 33, 20])),
    # two EP groups of two ranks inside a world of four (ranks 2, 3 are ranks 0, 1 of theirs)
    (4, dict(E=8, S=1, k=2, d=64, F=64, g=64, T=[20, 7, 13, 31], subgroups=True)),
    # fixed-capacity dispatch (no host copy of the counts): ragged and empty token counts,
    # shared experts, a rank receiving nothing, fine-grained routing
    (2, dict(E=8, S=0, k=2, d=64, F=64, g=64, T=[16, 16], dispatch="capacity", cap=16)),
    (2, dict(E=8, S=1, k=2, d=64, F=128, g=64, T=[5, 17], dispatch="capacity", cap=24)),
    (4, dict(E=8, S=0, k=3, d=64, F=64, g=64, T=[30, 0, 12, 1], dispatch="capacity", cap=32)),
    (4, dict(E=64, S=2, k=6, d=64, F=64, g=64, T=[9, 3, 8, 2], dispatch="capacity", cap=9)),
    # peer-memory exchange, restated on CPU ranks: decode-sized steps (send-back), a rank
    # with no tokens, fine-grained routing, and prefill-sized steps (the fused down path)
    (2, dict(E=8, S=0, k=2, d=64, F=64, g=64, T=[16, 16], dispatch="p2p", cap=16)),
    (4, dict(E=8, S=1, k=3, d=64, F=64, g=64, T=[30, 0, 12, 1], dispatch="p2p", cap=32)),
    (4, dict(E=64, S=2, k=6, d=64, F=64, g=64, T=[9, 3, 8, 2], dispatch="p2p", cap=9)),
    (2, dict(E=8, S=1, k=2, d=64, F=128, g=64, T=[290, 70], dispatch="p2p", cap=300)),
])
def test_expert_parallel_matches_single_process(world, case):
    results, codes = _run(world, case)
    assert len(results) == world, (results, codes)
    for r in range(world):
        status, val = results[r]
        assert status == "ok", val
        assert val <= 1e-5, f"rank {r}: max rel err {val}"


def test_rank_failure_is_reported_not_hung():
    case = dict(E=8, S=0, k=2, d=64, F=64, g=64, T=[16, 16], die=1)
    results, codes = _run(2, case, timeout=90)
    assert codes[1] == 3
    assert 0 in results and results[0][0] == "error", results


def test_slice_experts_rejects_ranges_outside_the_experts():
    from light_moe_b200.expert_parallel import slice_experts
    from light_moe_b200.layer import W4A16Experts
    E, S = 4, 1
    ex = W4A16Experts(torch.zeros((E + S) * 8, dtype=torch.uint8), torch.zeros((E + S) * 4, dtype=torch.uint8),
                      E, S, 128, 128, 128)
    part = slice_experts(ex, 2, 4)
    assert part.num_experts == 2 and part.num_shared == 1 and part.w13_packed.numel() == 3 * 8
    for e0, e1 in ((3, 5), (-1, 1), (3, 2)):
        with pytest.raises(ValueError):
            slice_experts(ex, e0, e1)
