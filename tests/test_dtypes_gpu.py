"""The drop-in ops on every floating dtype the reference's ops accept.

The reference's router converts hidden states and gate weight to fp32 and multiplies them in
fp32 (csrc/fused_moe_ops.cu:158-159); its grouped_gemm runs one GEMM per expert in the input
dtype (csrc/grouped_gemm.cu:24-40).  These tests call the same library entry points with
fp32, fp16 and mixed operands and check:
  * router: given the kernel's own fp32 logits, ids / weights / counts / offsets /
    sorted_idx are bit-identical to the oracle; the logits are within the fp32 accumulation
    bound of fp64 logits of the caller's values (not of bf16-rounded copies); every token
    whose top-k margin exceeds twice that bound selects exactly the fp64 oracle's experts --
    including the reference's own correctness case (fp32 [128, 4096], unit-variance gate,
    top-2, benchmarks/fused_ops_benchmark.py:108-140);
  * grouped_gemm: fp16 within fp16 output rounding of an fp32 reference, fp32 within fp32
    accumulation error, in the input dtype, through the C ABI and through the `_C` op.
"""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import dense_gemm, router

pytestmark = pytest.mark.gpu


def _check_given_logits(out, k, E):
    ids, w = oracle.route(out["logits"], k)
    assert np.array_equal(out["ids"], ids)
    assert np.array_equal(out["weights"].view(np.uint32), w.view(np.uint32)), "weights not bit-exact"
    counts, offsets, sidx = oracle.counts_offsets(ids, E)
    assert np.array_equal(out["counts"], counts)
    assert np.array_equal(out["offsets"], offsets)
    assert np.array_equal(out["sorted_idx"], sidx)


def _end_to_end(out, x, w, k, min_safe=0.95):
    xf = x.double().cpu().numpy()
    wf = w.double().cpu().numpy()
    lg64 = xf @ wf.T
    bound = (np.abs(xf) @ np.abs(wf).T) * 2.0 ** -18 + 1e-30
    assert np.all(np.abs(out["logits"] - lg64) <= bound), np.max(np.abs(out["logits"] - lg64) / bound)
    ids_ref, _ = oracle.route(lg64.astype(np.float32), k)
    srt = np.sort(lg64, axis=1)[:, ::-1]
    E = w.shape[0]
    safe = (srt[:, k - 1] - srt[:, k] > 2 * bound.max(axis=1)) if k < E else np.ones(x.shape[0], bool)
    assert safe.mean() >= min_safe, safe.mean()
    assert np.array_equal(np.sort(out["ids"][safe], 1), np.sort(ids_ref[safe], 1))
    return safe


def test_router_reference_fp32_check():
    """benchmarks/fused_ops_benchmark.py:108-140: fp32 hidden [128, 4096], fp32 randn gate [8, 4096], top-2."""
    g = torch.Generator(device="cpu").manual_seed(2024)
    x = torch.randn(128, 4096, generator=g).cuda()
    w = torch.randn(8, 4096, generator=g).cuda()
    out = router(x, w, 2)
    _check_given_logits(out, 2, 8)
    # the reference check's criterion is the same expert set as an fp32 GEMM + torch.topk; here
    # every token whose 2nd / 3rd logit gap exceeds twice the fp32 rounding bound (>= 99 % of
    # them) selects exactly the fp64 oracle's experts, and the rest are routed bit-exactly on
    # the kernel's own fp32 logits (checked above)
    _end_to_end(out, x, w, 2, min_safe=0.99)


@pytest.mark.parametrize("T,d,E,k,xdt,wdt", [
    (128, 4096, 8, 2, torch.float32, torch.float32),     # small-batch path, fp32
    (129, 256, 16, 4, torch.float32, torch.float32),     # first CUDA-core tiled size
    (5000, 1024, 64, 6, torch.float32, torch.float32),   # several tiles, E > 16
    (3000, 512, 8, 2, torch.float32, torch.bfloat16),    # mixed: fp32 hidden, bf16 gate
    (700, 256, 40, 7, torch.bfloat16, torch.float32),    # mixed: bf16 hidden, fp32 gate, ragged E
    (2000, 256, 8, 2, torch.float16, torch.bfloat16),    # fp16 with bf16: CUDA cores
    (40000, 128, 256, 16, torch.float32, torch.float32), # count table staged in several chunks
])
def test_router_non_bf16_inputs(T, d, E, k, xdt, wdt):
    g = torch.Generator(device="cpu").manual_seed(T + E)
    x = torch.randn(T, d, generator=g).to(xdt).cuda()
    w = (torch.randn(E, d, generator=g) * 0.05).to(wdt).cuda()
    out = router(x, w, k)
    _check_given_logits(out, k, E)
    _end_to_end(out, x, w, k)
    np.testing.assert_allclose(out["weights"].sum(1), np.ones(T), atol=1e-5)


@pytest.mark.parametrize("T,d,E,k", [(64, 4096, 8, 2), (1000, 512, 64, 6), (16384, 4096, 8, 2)])
def test_router_fp16_tensor_cores(T, d, E, k):
    g = torch.Generator(device="cpu").manual_seed(3 * T + E)
    x = torch.randn(T, d, generator=g).to(torch.float16).cuda()
    w = (torch.randn(E, d, generator=g) * 0.02).to(torch.float16).cuda()
    out = router(x, w, k)
    _check_given_logits(out, k, E)
    _end_to_end(out, x, w, k)


def test_router_op_keeps_the_callers_dtype():
    """_C.fused_gate_topk / fused_gate_topk_permute on fp32 input: fp32 weights out, the
    permuted rows are the caller's fp32 rows unchanged, ids from fp32 logits."""
    from light_moe_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(5)
    x = torch.randn(300, 256, generator=g).cuda()
    w = torch.randn(8, 256, generator=g).cuda()
    ids, wts = ops.fused_gate_topk(x, w, 2)
    assert ids.dtype == torch.int32 and wts.dtype == torch.float32
    perm, ids2, wts2, offs, sidx = ops.fused_gate_topk_permute(x, w, 2)
    assert perm.dtype == torch.float32 and offs.dtype == torch.int64 and sidx.dtype == torch.int64
    assert torch.equal(perm, x[sidx // 2])
    assert torch.equal(ids, ids2) and torch.equal(wts, wts2)
    out = router(x, w, 2)
    assert np.array_equal(ids.cpu().numpy(), out["ids"])
    h16 = x.half()
    ids16, w16 = ops.fused_gate_topk(h16, w.half(), 2)
    assert w16.dtype == torch.float16


def _segments(R, E, seed):
    rng = np.random.default_rng(seed)
    cuts = np.sort(rng.integers(0, R + 1, E - 1))
    return np.concatenate([[0], cuts, [R]]).astype(np.int64)


@pytest.mark.parametrize("dt,R,K,N,E", [(torch.float16, 700, 256, 192, 5), (torch.float16, 64, 4096, 512, 8),
                                        (torch.float32, 700, 260, 200, 5), (torch.float32, 33, 4096, 64, 3)])
def test_grouped_gemm_in_the_input_dtype(dt, R, K, N, E):
    g = torch.Generator(device="cpu").manual_seed(R + K)
    x = torch.randn(R, K, generator=g).to(dt).cuda()
    w = (torch.randn(E, N, K, generator=g) * 0.05).to(dt).cuda()
    off = _segments(R, E, R)
    offsets = torch.from_numpy(off).cuda()
    out = dense_gemm(x, w, offsets)
    assert out.dtype == dt
    ref = torch.zeros(R, N, dtype=torch.float64)
    xd, wd = x.double().cpu(), w.double().cpu()
    for e in range(E):
        a, b = int(off[e]), int(off[e + 1])
        ref[a:b] = xd[a:b] @ wd[e].T
    err = (out.double().cpu() - ref).abs()
    scale = ref.abs().max().item()
    if dt == torch.float16:
        # fp16 products are exact, fp32 accumulation, one fp16 rounding of the output
        assert (err <= ref.abs() * 2.0 ** -10 + 1e-3 * scale).all(), err.max().item()
    else:
        # sequential fp32 accumulation: |error| <= K * 2^-24 * sum_k |x||w|
        per_row = torch.zeros(R, N, dtype=torch.float64)
        for e in range(E):
            a, b = int(off[e]), int(off[e + 1])
            per_row[a:b] = xd[a:b].abs() @ wd[e].abs().T
        assert (err <= per_row * K * 2.0 ** -24 + 1e-30).all(), (err / (per_row + 1e-30)).max().item()
    # the `_C` op returns the same values in the same dtype
    from light_moe_b200 import ops
    out2 = ops.grouped_gemm(x, w, offsets, E)
    assert out2.dtype == dt and torch.equal(out2, out)
