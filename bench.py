"""Benchmark: W4A16 MoE-layer tokens/s on B200 (Mixtral-8x7B expert shapes).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1: expert parallel over NCCL)

Workload (one "step" = one forward of the MoE layer over one batch):
  d=4096, ffn=14336, 8 SwiGLU experts, top-2, int4 weights (symmetric, group 128, fp16
  scales) quantised from N(0, 0.02); router N(0, 0.02) bf16; x ~ N(0, 1) bf16; seeded.
  Headline: prefill, 8192 tokens per GPU.  A decode sub-measurement (64 tokens per GPU)
  is reported under "decode".
Timing: CUDA events on the launching stream, barrier + synchronize on both sides, max over
ranks.  The int4 weights (727 MB) exceed the 126 MB L2, so every step streams them from HBM.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

D, FFN, E, TOPK, GROUP = 4096, 14336, 8, 2, 128
METRIC = "W4A16 MoE-layer tokens/s (Mixtral-8x7B experts, prefill 8192 tokens/GPU)"
T_PREFILL, T_DECODE = 8192, 64
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", f"lmoe_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx = float(parts[2])
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- problem
def make_problem(T, device, seed=0):
    import torch
    from light_moe_b200.layer import W4A16Experts

    g = torch.Generator(device=device).manual_seed(seed)
    gw = (torch.randn(E, D, generator=g, device=device) * 0.02).to(torch.bfloat16)
    # quantise expert by expert to bound the transient bf16 footprint
    q1s, s1s, q3s, s3s, q2s, s2s = [], [], [], [], [], []
    from light_moe_b200 import ops
    for e in range(E):
        w1 = (torch.randn(FFN, D, generator=g, device=device) * 0.02).to(torch.bfloat16)
        w3 = (torch.randn(FFN, D, generator=g, device=device) * 0.02).to(torch.bfloat16)
        w2 = (torch.randn(D, FFN, generator=g, device=device) * 0.02).to(torch.bfloat16)
        for (w, qs, ss) in ((w1, q1s, s1s), (w3, q3s, s3s), (w2, q2s, s2s)):
            q, s = ops.quantize_w4(w, GROUP)
            qs.append(q)
            ss.append(s)
        del w1, w3, w2
    st = torch.stack
    ex = W4A16Experts.from_quantized(st(q1s), st(s1s), st(q3s), st(s3s), st(q2s), st(s2s), E, GROUP,
                                     keep_canonical=True)
    gx = torch.Generator(device=device).manual_seed(seed + 1)
    x = torch.randn(T, D, generator=gx, device=device).to(torch.bfloat16)
    return x, gw, ex


def l2_note(ex, ws, T):
    """How the timed steps relate to the 126 MB L2, per rank."""
    w = (ex.w13_packed.numel() + ex.w2_packed.numel()) / ws / 1e6
    act = T * TOPK * (D + FFN) * 2 / 1e6   # dispatched rows and the SwiGLU output, bf16
    if w > 126:
        return f"inputs larger than L2: {w:.0f} MB of int4 weights per GPU streamed every step"
    return (f"{w:.0f} MB of int4 weights per GPU fit in the 126 MB L2, but every step also streams "
            f"~{act:.0f} MB of dispatched rows and SwiGLU output per GPU, which evicts them")


# ----------------------------------------------------------------------------- timing helpers
def time_device(fn, steps, warmup, stream, barrier=None):
    import torch
    for _ in range(warmup):
        fn()
    if barrier:
        barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        fn()
    ev1.record(stream)
    torch.cuda.synchronize()
    if barrier:
        barrier()
    return ev0.elapsed_time(ev1) / 1e3  # seconds


def time_host_calls(layer, xh, yh, steps, warmup, stream, barrier=None):
    """Device seconds of `steps` back-to-back host-buffer layer calls
    (W4A16MoELayer.forward_host_async: each call's input copies run beside the previous
    call's kernels, its output copies beside the next call's).  The timed region opens before
    the first call's input copy and closes after the last call's output copy, so every
    step's copies and kernels lie inside it."""
    import torch
    done = None
    for _ in range(warmup):
        _, done = layer.forward_host_async(xh, out=yh)
    if done is not None:
        done.synchronize()
    torch.cuda.synchronize()
    if barrier:
        barrier()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    streams = getattr(layer, "_copy_streams", None)
    if streams is not None:
        streams[0].wait_event(ev0)           # the first input copy starts after ev0
    for _ in range(steps):
        _, done = layer.forward_host_async(xh, out=yh)
    stream.wait_event(done)                  # ... and ev1 after the last output copy
    ev1.record(stream)
    torch.cuda.synchronize()
    if barrier:
        barrier()
    return ev0.elapsed_time(ev1) / 1e3


def time_graph(fn, calls, replays, stream):
    """Device seconds per call of `fn`, from `calls` calls captured in one CUDA graph and
    replayed `replays` times: the launches cost no host time, so a kernel shorter than its
    host-side call overhead is still timed on the device alone."""
    import torch
    fn()
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        for _ in range(calls):
            fn()
    graph.replay()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(replays):
        graph.replay()
    ev1.record(stream)
    torch.cuda.synchronize()
    del graph
    return ev0.elapsed_time(ev1) / 1e3 / (calls * replays)


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of the roofline
# kernel, from ncu captures of this bench's own workloads: the gate/up GEMM at T=8192 (first
# launch of the first layer call, 623.8 MB read + 442.0 MB written) and the decode gate/up
# GEMM at T=64 (485.6 MB read + 7.4 MB written).  Other sizes report null.
NCU_TRAFFIC_BYTES = {8192: 623760128 + 441977088, 64: 485.6e6 + 7.4e6}


def gemm_roofline(x, gw, ex, T, stream, peaks, peak_kind):
    """Time the dominant kernel (gate/up W4A16 GEMM, SwiGLU epilogue) alone on its stream."""
    import torch
    from light_moe_b200 import ops

    ids, wts, counts, offsets, sidx = ops.fused_gate_topk_ex(x, gw, TOPK)[:5]
    xp = x[(sidx // TOPK).long()].contiguous()
    R = T * TOPK

    def run():
        return ops.w4a16_grouped_gemm(xp, ex.w13_packed, offsets, E, 2 * FFN, GROUP, 1, None, None, 0, T)

    launches = 20
    secs = time_device(run, launches, 3, stream) / launches
    flops = 2.0 * R * (2 * FFN) * D
    bytes_ = ex.w13_packed.numel() + R * D * 2 + R * FFN * 2
    if T >= 1024:
        achieved = flops / secs / 1e12
        peak = peaks["bf16_tflops"]
        return {"kernel": "grouped_gemm_kernel<192,...,W4> gate/up+SwiGLU", "bound": "tensor",
                "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                "peak_source": f"{peak_kind} bf16 burst", "launch_us": round(secs * 1e6, 1),
                "algorithmic": {"flops": flops, "bytes": bytes_}, "traffic": NCU_TRAFFIC_BYTES.get(T),
                "traffic_unit": "DRAM bytes per launch (ncu)"}
    achieved = bytes_ / secs / 1e9
    peak = peaks["hbm_gbs"]
    return {"kernel": "w4_decode_kernel gate/up+SwiGLU", "bound": "hbm",
            "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
            "peak_source": f"{peak_kind} HBM copy", "launch_us": round(secs * 1e6, 1),
            "algorithmic": {"flops": flops, "bytes": bytes_}, "traffic": NCU_TRAFFIC_BYTES.get(T),
            "traffic_unit": "DRAM bytes per launch (ncu)"}


# ----------------------------------------------------------------------------- other workloads
def extra_workloads(ex, stream, peaks, peak_kind, device):
    """Single-GPU measurements of the other workloads of the hot path (reported beside the
    headline, never folded into it): the router alone, the Mixtral grouped GEMMs with a
    skewed expert load, and the fine-grained 64-expert layer."""
    import torch

    from light_moe_b200 import ops
    from light_moe_b200.layer import W4A16Experts, W4A16MoELayer

    out = {}
    g = torch.Generator(device=device).manual_seed(0)
    # router: x [16384, 4096] bf16, W [E, 4096]; HBM-bound on the x stream.  Right after the
    # GEMM-heavy measurements the GPU runs memory-bound kernels ~15 % slower for a few seconds
    # (the router alone: 35 us after an idle pause, 41 us straight after 20 prefill layers), so
    # the router is timed after a 3 s pause, like a kernel timed on its own
    T = 16384
    x = torch.randn(T, D, generator=g, device=device).to(torch.bfloat16)
    torch.cuda.synchronize()
    time.sleep(3.0)
    router = []
    for e, k in ((8, 2), (64, 6)):
        w = (torch.randn(e, D, generator=g, device=device) * 0.02).to(torch.bfloat16)
        # device time per call (graph replay); the eager call also pays ~10-40 us of host time
        secs = time_graph(lambda: ops.fused_gate_topk_ex(x, w, k), 20, 5, stream)
        eager = time_device(lambda: ops.fused_gate_topk_ex(x, w, k), 20, 3, stream) / 20
        nbytes = T * D * 2 + e * D * 2 + T * k * 16 + (2 * e + 1) * 4   # x, W; ids, weights, sorted_idx, positions
        gbs = nbytes / secs / 1e9
        router.append({"experts": e, "top_k": k, "tokens": T, "us": round(secs * 1e6, 1), "GB/s": round(gbs, 1),
                       "frac_of_hbm": round(gbs / peaks["hbm_gbs"], 4), "algorithmic_bytes": nbytes,
                       "timing": "CUDA graph of 20 calls, after a 3 s idle pause", "eager_us": round(eager * 1e6, 1)})
    out["router"] = router
    del x
    # grouped GEMMs (gate/up + SwiGLU, down) over 8192 rows, Zipf(1.2) expert load
    R = 8192
    p = [(i + 1) ** -1.2 for i in range(E)]
    cnt = [int(R * v / sum(p)) for v in p]
    cnt[0] += R - sum(cnt)
    offs = torch.tensor([0] + [sum(cnt[:i + 1]) for i in range(E)], dtype=torch.int32, device=device)
    xr = torch.randn(R, D, generator=g, device=device).to(torch.bfloat16)

    def gemms():
        h = ops.w4a16_grouped_gemm(xr, ex.w13_packed, offs, E, 2 * FFN, GROUP, 1, None, None, 0, max(cnt))
        return ops.w4a16_grouped_gemm(h, ex.w2_packed, offs, E, D, GROUP, 0, None, None, 0, max(cnt))

    secs = time_device(gemms, 10, 3, stream) / 10
    flops = 2.0 * R * 3 * D * FFN
    out["grouped_gemm_zipf"] = {"rows": R, "rows_per_expert": cnt, "ms": round(secs * 1e3, 4),
                                "TFLOP/s": round(flops / secs / 1e12, 1),
                                "frac_of_bf16_peak": round(flops / secs / 1e12 / peaks["bf16_tflops"], 4)}
    del xr
    # fine-grained layer: d=2048, 64 routed experts (ffn 1408) top-6 + 2 shared, int4 g=64
    d5, f5, e5, k5, s5, g5, t5 = 2048, 1408, 64, 6, 2, 64, 16384
    w1 = (torch.randn(e5 + s5, f5, d5, generator=g, device=device) * 0.02).to(torch.bfloat16)
    w3 = (torch.randn(e5 + s5, f5, d5, generator=g, device=device) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(e5 + s5, d5, f5, generator=g, device=device) * 0.02).to(torch.bfloat16)
    shared = [(w1[e5 + i], w3[e5 + i], w2[e5 + i]) for i in range(s5)]
    ex5 = W4A16Experts.from_dense(w1[:e5], w3[:e5], w2[:e5], g5, shared=shared)
    del w1, w3, w2
    gw5 = (torch.randn(e5, d5, generator=g, device=device) * 0.02).to(torch.bfloat16)
    bias5 = torch.linspace(0.5, -0.5, e5, device=device)   # skews the load toward low ids
    layer5 = W4A16MoELayer(gw5, ex5, k5, gate_bias=bias5)
    x5 = torch.randn(t5, d5, generator=g, device=device).to(torch.bfloat16)
    secs = time_device(lambda: layer5(x5), 10, 3, stream) / 10
    flops = 2.0 * t5 * (k5 + s5) * 3 * d5 * f5
    out["fine_grained_layer"] = {"tokens": t5, "hidden": d5, "ffn": f5, "experts": e5, "top_k": k5, "shared": s5,
                                 "group_size": g5, "ms": round(secs * 1e3, 4), "tokens/s": round(t5 / secs, 1),
                                 "TFLOP/s": round(flops / secs / 1e12, 1),
                                 "frac_of_bf16_peak": round(flops / secs / 1e12 / peaks["bf16_tflops"], 4)}
    out["peak_source"] = peak_kind
    return out


# ----------------------------------------------------------------------------- CPU reference path
def host_threads():
    """(logical cores of the host, threads torch uses for CPU math)."""
    import torch
    return os.cpu_count(), torch.get_num_threads()


def reference_block():
    """The reference's own SparseMoEBlock (python/light_moe/model/moe_block.py:63-169) at the
    layer's shapes, fp32 on the host, when its bytecode is staged under oracle/_ref
    (oracle/stage_reference.py); else None."""
    import torch

    from oracle.stage_reference import available, import_sparse_moe_block
    if not available():
        return None
    SparseMoEBlock = import_sparse_moe_block()
    torch.manual_seed(0)
    blk = SparseMoEBlock(D, FFN, num_experts=E, top_k=TOPK).eval()
    # N(0, 0.02) weights like the GPU workload (the values do not change the CPU work; the
    # dequantised int4 values are N(0, 0.02) samples rounded to the int4 grid)
    with torch.no_grad():
        for prm in blk.parameters():
            prm.normal_(0.0, 0.02)
    return blk


def time_reference_block(blk, tokens, steps, warmup, budget_s):
    """Seconds per forward of ``blk`` on ``tokens`` tokens (torch fp32, all host threads).
    Returns (seconds per step, steps timed): after one warm-up forward, fewer than ``steps``
    are timed when ``steps`` of them would exceed ``budget_s``."""
    import torch
    x = torch.randn(1, tokens, D, generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        t0 = time.perf_counter()
        blk(x)
        first = time.perf_counter() - t0
        for _ in range(max(0, warmup - 1) if first * warmup < budget_s / 4 else 0):
            blk(x)
        n = max(1, min(steps, int(budget_s // max(first, 1e-6))))
        t0 = time.perf_counter()
        for _ in range(n):
            blk(x)
        el = time.perf_counter() - t0
    return el / n, n


def cpu_baseline(ex, gw, tokens, seconds_budget=20.0):
    """The reference's own SparseMoEBlock on the host cores (oracle restatement if it is not
    staged), on a bounded sample of the workload."""
    import numpy as np

    cores, threads = host_threads()
    blk = reference_block()
    if blk is not None:
        secs, n = time_reference_block(blk, tokens, 1000, 1, seconds_budget)
        del blk
        return {"value": round(tokens / secs, 2), "unit": "tokens/s", "cores": threads, "host_cores": cores,
                "kind": "reference",
                "sample": f"{n} forward(s) of light_moe SparseMoEBlock (fp32, torch, {threads} threads) on "
                          f"{tokens} tokens of the layer"}
    import oracle
    from light_moe_b200 import ops

    c = ex.canonical
    w1 = ops.dequantize_w4(c["q1"], c["s1"], GROUP).float().cpu().numpy()
    w3 = ops.dequantize_w4(c["q3"], c["s3"], GROUP).float().cpu().numpy()
    w2 = ops.dequantize_w4(c["q2"], c["s2"], GROUP).float().cpu().numpy()
    gwn = gw.float().cpu().numpy()
    x = np.random.default_rng(1).standard_normal((tokens, D), dtype=np.float32)
    oracle.moe_layer_ref(x[:8], gwn, w1, w3, w2, TOPK)  # warm-up
    done, reps, t0 = 0, 0, time.perf_counter()
    while True:
        oracle.moe_layer_ref(x, gwn, w1, w3, w2, TOPK)
        done += tokens
        reps += 1
        el = time.perf_counter() - t0
        if el > seconds_budget or reps >= 3:
            break
    return {"value": round(done / el, 2), "unit": "tokens/s", "cores": threads, "host_cores": cores, "kind": "port",
            "sample": f"{reps} x {tokens} tokens through the fp32 numpy SparseMoEBlock restatement"}


# ----------------------------------------------------------------------------- arms
def measure_decode(args, x, gw, ex, layer, ws, stream, barrier, peaks, peak_kind, device):
    """Decode step (64 tokens per GPU), on every rank.  One GPU: the single-GPU layer; N GPUs:
    the expert-parallel layer with fixed-capacity dispatch (no host synchronisation).  The
    step is timed eagerly and as a CUDA graph replay (how a serving loop runs decode); the
    reported step time is the replay's, max over ranks."""
    import torch
    import torch.distributed as dist

    from light_moe_b200.layer import W4A16MoELayer
    xd = x[:T_DECODE].contiguous()
    # a decode loop is memory-bound and runs at a lower power level than the prefill GEMMs
    # timed just before; memory-bound kernels run ~15 % slower for a few seconds after those,
    # so the decode step is timed after a 3 s pause
    torch.cuda.synchronize()
    time.sleep(3.0)
    check = None
    if ws > 1:
        from light_moe_b200.expert_parallel import ExpertParallelW4A16Layer
        dmode = "p2p" if args.ep_dispatch == "p2p" else "capacity"
        dlayer = ExpertParallelW4A16Layer.from_full(gw, ex, TOPK, group=None, dispatch=dmode,
                                                    capacity_tokens=T_DECODE)
        y_ep = dlayer(xd)
        y_one = W4A16MoELayer(gw, ex, TOPK)(xd)
        rel = ((y_ep.float() - y_one.float()).abs().max() / y_one.float().abs().max()).double().reshape(1)
        dist.all_reduce(rel, op=dist.ReduceOp.MAX)
        check = float(rel.item())
        dfwd = dlayer.forward
    else:
        dfwd = layer.forward
    dsteps = max(args.steps, 20)
    eager = time_device(lambda: dfwd(xd), dsteps, args.warmup, stream, barrier) / dsteps
    if barrier:
        barrier()
    graph = time_graph(lambda: dfwd(xd), 10, max(2, dsteps // 10), stream)
    t = torch.tensor([eager, graph], device=device, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    eager, graph = float(t[0]), float(t[1])
    wbytes = (ex.w13_packed.numel() + ex.w2_packed.numel()) / ws
    layer_gbs = wbytes / graph / 1e9
    out = {"tokens_per_gpu": T_DECODE, "value": round(T_DECODE * ws / graph, 1), "unit": "tokens/s",
           "ms_per_step": round(graph * 1e3, 4), "eager_ms_per_step": round(eager * 1e3, 4),
           "timing": "CUDA graph replay of 10 steps (max over ranks), after a 3 s idle pause; eager: back-to-back calls",
           "dispatch": ("single GPU" if ws == 1 else
                        "peer-memory copies (NVLink), no NCCL and no host synchronisation" if args.ep_dispatch == "p2p"
                        else "fixed-capacity NCCL all-to-all, no host synchronisation"),
           "layer_weight_stream_gbs_per_gpu": round(layer_gbs, 1),
           "layer_frac_of_hbm": round(layer_gbs / peaks["hbm_gbs"], 4)}
    if ws > 1:
        out["ep_max_rel_err"] = check
        dlayer.close()
    else:
        out["roofline_gate_up"] = gemm_roofline(xd, gw, ex, T_DECODE, stream, peaks, peak_kind)
    return out


def run_ours(args):
    import torch
    import torch.distributed as dist

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if ws > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
        barrier = dist.barrier
    else:
        barrier = None
    peaks, peak_kind = load_peaks()
    stream = torch.cuda.current_stream()
    from light_moe_b200 import ops
    from light_moe_b200.layer import W4A16MoELayer

    T = args.tokens
    x, gw, ex = make_problem(T, device, seed=0)
    if ws > 1:
        from light_moe_b200.expert_parallel import ExpertParallelW4A16Layer
        if args.ep_dispatch == "p2p":
            layer = ExpertParallelW4A16Layer.from_full(gw, ex, TOPK, group=None, dispatch="p2p", capacity_tokens=T)
            # router, counts exchange, dispatch, wait, gate/up GEMM, down GEMM, send-back, wait, combine
            launches_per_step = 9
        else:
            layer = ExpertParallelW4A16Layer.from_full(gw, ex, TOPK, group=None, micro_batches=args.micro_batches,
                                                       sm_reserve=args.sm_reserve)
            launches_per_step = 5 * layer.micro_batches
        fwd = layer.forward
    else:
        layer = W4A16MoELayer(gw, ex, TOPK)
        fwd = layer.forward
        launches_per_step = 6   # router, table, gather, gate/up GEMM, down GEMM, combine

    def step():
        return fwd(x)

    with ClockSampler(local) as clk:
        secs = time_device(step, args.steps, args.warmup, stream, barrier)
    # max over ranks
    t = torch.tensor([secs], device=device, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    secs = t.item()
    value = T * ws * args.steps / secs

    # end to end through the public API: pinned host x -> device, layer, y -> pinned host,
    # with the layer's asynchronous host-buffer calls back to back (one GPU and expert
    # parallel alike): a call's copies overlap the neighbouring calls' kernels.
    xh = x.cpu().pin_memory()
    yh = torch.empty_like(xh).pin_memory()

    esecs = time_host_calls(layer, xh, yh, args.steps, args.warmup, stream, barrier)
    te = torch.tensor([esecs], device=device, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = T * ws * args.steps / te.item()

    ep_check = None
    roof_ep = None
    if ws > 1:
        # parity of the expert-parallel step on every rank: its output against the
        # single-GPU layer (all experts on this GPU) on the rank's own tokens
        y_ep = fwd(x)
        y_one = W4A16MoELayer(gw, ex, TOPK)(x)
        rel = ((y_ep.float() - y_one.float()).abs().max() / y_one.float().abs().max()).double().reshape(1)
        dist.all_reduce(rel, op=dist.ReduceOp.MAX)
        ep_check = float(rel.item())
        # the per-rank gate/up GEMM inside the expert-parallel step (events around the launch)
        layer.backend.gemm_timer = []
        for _ in range(3):
            fwd(x)
        torch.cuda.synchronize()
        times = [(a.elapsed_time(b) / 1e3, rows) for a, b, rows in layer.backend.gemm_timer]
        layer.backend.gemm_timer = None
        g_secs = sum(t for t, _ in times) / len(times)
        g_rows = sum(r for _, r in times) / len(times)
        tf = 2.0 * g_rows * (2 * FFN) * D / g_secs / 1e12
        agg = torch.tensor([tf, -tf], device=device, dtype=torch.float64)
        dist.all_reduce(agg, op=dist.ReduceOp.MAX)
        roof_ep = {"kernel": "grouped_gemm_kernel<192,...,W4> gate/up+SwiGLU (this rank's experts, inside the EP step)",
                   "bound": "tensor", "achieved": round(tf, 1), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                   "frac": round(tf / peaks["bf16_tflops"], 4), "peak_source": f"{peak_kind} bf16 burst",
                   "launch_us": round(g_secs * 1e6, 1), "rows": round(g_rows, 1),
                   "ranks_max_tflops": round(agg[0].item(), 1), "ranks_min_tflops": round(-agg[1].item(), 1),
                   "algorithmic": {"flops": 2.0 * g_rows * (2 * FFN) * D}, "traffic": None,
                   "traffic_unit": "DRAM bytes per launch (ncu); not captured for the per-rank launch"}

    decode_all = measure_decode(args, x, gw, ex, layer if ws == 1 else None, ws, stream, barrier, peaks, peak_kind,
                                device)

    result = None
    if rank == 0:
        roof = roof_ep if ws > 1 else gemm_roofline(x, gw, ex, T, stream, peaks, peak_kind)
        decode = decode_all
        extra = None
        if ws == 1 and not args.no_extra:
            try:
                extra = extra_workloads(ex, stream, peaks, peak_kind, device)
            except Exception as exc:   # reported, never hides the headline line
                extra = {"error": f"{type(exc).__name__}: {exc}"}
        cpu = None
        if not args.no_cpu_baseline and ws == 1:   # the CPU baseline is a single-GPU (rank 0, N=1) figure
            cpu = cpu_baseline(ex, gw, args.cpu_tokens)
        result = {
            "metric": METRIC,
            "value": round(value, 1), "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(secs / args.steps * 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16 activations, int4 weights, fp32 accumulate",
            "data": "synthetic (seeded N(0,1) tokens, N(0,0.02) weights quantised to int4)",
            "config": {"workload": "Mixtral-8x7B-shaped W4A16 MoE layer, prefill", "tokens_per_gpu": T,
                       "hidden": D, "ffn": FFN, "experts": E, "top_k": TOPK, "group_size": GROUP,
                       "parallelism": f"ep{ws}" if ws > 1 else "single GPU",
                       "ep_dispatch": (None if ws == 1 else "peer-memory copies over NVLink (no NCCL on the data path)"
                                       if args.ep_dispatch == "p2p" else "NCCL all-to-all-v"),
                       "ep_micro_batches": args.micro_batches if ws > 1 and args.ep_dispatch != "p2p" else None,
                       "ep_sm_reserve": layer.sm_reserve if ws > 1 else None,
                       "l2": l2_note(ex, ws, T)},
            "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s", "h2d_bytes_per_step": T * D * 2,
                    "d2h_bytes_per_step": T * D * 2,
                    "call": ("W4A16MoELayer.forward_host_async called back to back (pinned host buffers; a call's "
                             "input / output copies overlap the previous / next call's kernels); timed from "
                             "before the first input copy to after the last output copy" if ws == 1 else
                             "ExpertParallelW4A16Layer.forward_host_async called back to back on every rank "
                             "(pinned host buffers, one token range per call, copies beside the neighbouring "
                             "calls' kernels); max over ranks")},
            "gpu_launches": launches_per_step * args.steps,
            "ep_max_rel_err": ep_check,
            "roofline": roof,
            "decode": decode,
            "other_workloads": extra,
            "cpu_baseline": cpu,
            "clocks": clk.summary(),
        }
        print(json.dumps(result), flush=True)
    if ws > 1:
        if hasattr(layer, "close"):
            layer.close()
        dist.barrier()
        dist.destroy_process_group()
    return result


def run_reference(args):
    """CPU arm: light-moe's own SparseMoEBlock (staged bytecode of the reference package) in
    fp32 torch on the host cores, on the headline workload (8192 tokens per step); the
    oracle's numpy restatement when the reference is not staged."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return None
    import numpy as np

    cores, threads = host_threads()
    tokens = args.tokens
    blk = reference_block()
    budget = 180.0
    if blk is not None:
        secs, n = time_reference_block(blk, tokens, args.steps, args.warmup, budget)
        kind = "reference"
        sample = (f"light_moe SparseMoEBlock.forward (python/light_moe/model/moe_block.py:119-169), fp32 torch, "
                  f"{threads} threads, {tokens} tokens per step, {n} timed step(s)")
    else:
        import oracle
        rng = np.random.default_rng(0)
        gw = (rng.standard_normal((E, D), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        w = {name: (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02))
             for name, shape in (("w1", (E, FFN, D)), ("w3", (E, FFN, D)), ("w2", (E, D, FFN)))}
        x = rng.standard_normal((tokens, D), dtype=np.float32)
        t0 = time.perf_counter()
        oracle.moe_layer_ref(x, gw, w["w1"], w["w3"], w["w2"], TOPK)
        first = time.perf_counter() - t0
        n = max(1, min(args.steps, int(budget // max(first, 1e-6))))
        t0 = time.perf_counter()
        for _ in range(n):
            oracle.moe_layer_ref(x, gw, w["w1"], w["w3"], w["w2"], TOPK)
        secs = (time.perf_counter() - t0) / n
        kind = "port"
        sample = f"oracle numpy restatement of SparseMoEBlock, {tokens} tokens per step, {n} timed step(s)"
    value = tokens / secs
    res = {"impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": ws,
           "steps": n, "warmup": args.warmup, "ms_per_step": round(secs * 1e3, 3), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (host)", "data": "synthetic (seeded)",
           "config": {"workload": "Mixtral-8x7B-shaped MoE layer, prefill", "tokens_per_step": tokens,
                      "hidden": D, "ffn": FFN, "experts": E, "top_k": TOPK, "group_size": GROUP},
           "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": threads, "host_cores": cores,
                            "kind": kind, "sample": sample},
           "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(res), flush=True)
    return res


KERNEL_CASES = ("router-e8", "router-e64", "gateup-t8192", "down-t8192", "decode-gateup-t64", "decode-down-t64")


def run_kernel_case(args):
    """One kernel of the path, launched `steps` times on the bench's inputs (for profiler
    captures of a single kernel; prints the CUDA-event time per launch)."""
    import torch

    from light_moe_b200 import ops
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    stream = torch.cuda.current_stream()
    case = args.kernel_case
    if case.startswith("router"):
        e, k = (8, 2) if case == "router-e8" else (64, 6)
        g = torch.Generator(device=device).manual_seed(0)
        x = torch.randn(16384, D, generator=g, device=device).to(torch.bfloat16)
        w = (torch.randn(e, D, generator=g, device=device) * 0.02).to(torch.bfloat16)
        fn = lambda: ops.fused_gate_topk_ex(x, w, k)   # noqa: E731
    else:
        T = 8192 if case.endswith("t8192") else T_DECODE
        x, gw, ex = make_problem(T, device, seed=0)
        ids, wts, counts, offsets, sidx = ops.fused_gate_topk_ex(x, gw, TOPK)[:5]
        xp = x[(sidx // TOPK).long()].contiguous()
        h = ops.w4a16_grouped_gemm(xp, ex.w13_packed, offsets, E, 2 * FFN, GROUP, 1, None, None, 0, T)
        if "gateup" in case:
            fn = lambda: ops.w4a16_grouped_gemm(xp, ex.w13_packed, offsets, E, 2 * FFN, GROUP, 1,  # noqa: E731
                                                None, None, 0, T)
        else:
            fn = lambda: ops.w4a16_grouped_gemm(h, ex.w2_packed, offsets, E, D, GROUP, 0,  # noqa: E731
                                                None, None, 0, T)
    secs = time_device(fn, args.steps, args.warmup, stream) / args.steps
    print(json.dumps({"kernel_case": case, "launches": args.steps + args.warmup, "us_per_launch": round(secs * 1e6, 1)}),
          flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=T_PREFILL)
    ap.add_argument("--cpu-tokens", type=int, default=1024)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the router / skewed-GEMM / fine-grained measurements")
    ap.add_argument("--ep-dispatch", choices=["p2p", "exact"], default="p2p",
                    help="N > 1: rows through peer memory (default) or NCCL all-to-alls (exact prefill, "
                         "fixed-capacity decode)")
    ap.add_argument("--micro-batches", type=int, default=1,
                    help="expert-parallel runs: micro-batches whose all-to-alls overlap the GEMMs")
    ap.add_argument("--sm-reserve", type=int, default=None,
                    help="expert-parallel runs: SMs the GEMMs leave to the all-to-alls (default 16 with "
                         "several micro-batches, else 0)")
    ap.add_argument("--kernel-case", choices=KERNEL_CASES, default=None,
                    help="launch one kernel of the path `steps` times (profiler captures) and exit")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.kernel_case:
        run_kernel_case(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
