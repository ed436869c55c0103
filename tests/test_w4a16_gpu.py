"""GPU parity of the int4 format kernels and the grouped GEMMs.

* quantise / dequantise: bit-exact against the CPU oracle;
* the GEMM's in-kernel dequantisation: bit-exact, read back through identity activations;
* GEMM results: against a plain PyTorch fp32 computation on the dequantised weights, with
  the tolerance of a bf16 output (relative 2^-7 of the row scale plus accumulation slack).
"""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import bf16_bits, bf16_gemm, dequantize, prepack, quantize, w4_gemm

pytestmark = pytest.mark.gpu

TOL = 1e-2  # max |y - y_ref| / max |y_ref|


def _w(shape, seed, scale=0.02, dtype=torch.bfloat16):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype).cuda()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("g", [64, 128])
def test_quantize_dequantize_bitexact(dtype, g):
    w = _w((3, 96, 512), seed=g, dtype=dtype)
    # plant exact half-way quotients: with max|w| = 7 the scale is 1 and w/s = n + 0.5
    w[0, 0, :8] = torch.tensor([7.0, -7.0, 2.5, 3.5, -2.5, -3.5, 0.5, -0.5], dtype=dtype)
    q, s = quantize(w, g)
    qo, so = oracle.quantize_w4(w.float().cpu().numpy(), g)
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.array_equal(s.view(torch.int16).cpu().numpy().view(np.uint16), so)
    deq = dequantize(q, s, g)
    assert np.array_equal(bf16_bits(deq), oracle.dequantize_w4(qo, so, g))


def test_quantize_zero_groups():
    w = torch.zeros(2, 128, 256, dtype=torch.bfloat16, device="cuda")
    q, s = quantize(w, 128)
    assert torch.all(q == 0x88) and torch.all(s == 0)
    assert torch.all(dequantize(q, s, 128) == 0)


def _expert_setup(E, N, K, g, seed, paired=False):
    w = _w((E, N, K), seed)
    q, s = quantize(w, g)
    deq = dequantize(q, s, g).float()
    if paired:
        w3 = _w((E, N, K), seed + 1)
        q3, s3 = quantize(w3, g)
        deq3 = dequantize(q3, s3, g).float()
        packed = prepack(q, s, g, q3, s3)
        return packed, deq, deq3
    packed = prepack(q, s, g)
    return packed, deq


def _offsets(counts, dtype=torch.int32):
    off = np.zeros(len(counts) + 1, np.int64)
    off[1:] = np.cumsum(counts)
    return torch.tensor(off, dtype=dtype, device="cuda")


def _ref_plain(x, deq, offsets):
    off = offsets.cpu().tolist()
    y = torch.zeros(x.shape[0], deq.shape[1], device="cuda")
    for e in range(len(off) - 1):
        a, b = off[e], off[e + 1]
        if b > a:
            y[a:b] = x[a:b].float() @ deq[e].T
    return y


def _assert_close(y, ref):
    err = (y.float() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= TOL * scale, (err, scale)
    # elementwise: bf16 rounding of the output plus fp32 accumulation slack
    assert torch.all((y.float() - ref).abs() <= ref.abs() * 2 ** -7 + 2e-3 * scale)


@pytest.mark.parametrize("K,g,hint", [(256, 128, 0), (4096, 128, 0), (2048, 64, 0), (4096, 128, 64), (2048, 64, 64)])
def test_gemm_dequant_bitexact_via_identity(K, g, hint):
    """X = identity rows: Y[r, n] = W_deq[n, r] exactly.  hint=0 runs the tcgen05 kernel
    (bf16 weights in tensor memory, one-term fp32 sums); hint=64 runs the decode kernel
    (integer weights, fp32 q*s applied after the MMA, one bf16 rounding at the output)."""
    E, N = 2, 256
    packed, deq = _expert_setup(E, N, K, g, seed=K + hint)
    rows = 64 if hint else min(K, 512)
    for r0 in range(0, min(K, 512), rows):
        eye = torch.eye(K, dtype=torch.bfloat16, device="cuda")[r0:r0 + rows]
        x = torch.cat([eye, eye])                   # expert 0 and expert 1 see the same rows
        off = _offsets([rows, rows])
        y = w4_gemm(x, packed, N, g, off, hint=hint)
        want0 = deq[0][:, r0:r0 + rows].T.to(torch.bfloat16)
        want1 = deq[1][:, r0:r0 + rows].T.to(torch.bfloat16)
        assert np.array_equal(bf16_bits(y[:rows]), bf16_bits(want0))
        assert np.array_equal(bf16_bits(y[rows:]), bf16_bits(want1))
        if not hint:
            break


@pytest.mark.parametrize("counts,hint", [
    ([100, 0, 37, 300, 1, 16, 17, 250], 0),
    ([5, 9, 16, 3, 0, 12, 7, 11], 64),
    ([16] * 8, 64),
    ([700, 500], 0),
])
def test_w4_gemm_plain(counts, hint):
    E, N, K, g = len(counts), 384, 512, 128
    packed, deq = _expert_setup(E, N, K, g, seed=sum(counts))
    R = sum(counts)
    x = _w((R, K), seed=R, scale=1.0)
    off = _offsets(counts)
    y = w4_gemm(x, packed, N, g, off, hint=hint)
    _assert_close(y, _ref_plain(x, deq, off))


@pytest.mark.parametrize("hint", [0, 64])
def test_w4_gemm_hole_segments(hint):
    """Segments mapped to weight matrix -1 (the padding of a fixed-capacity exchange) are
    skipped without an error and their output rows are left untouched; the other segments
    use their mapped matrices (several segments may share one)."""
    E, N, K, g = 3, 256, 512, 128
    packed, deq = _expert_setup(E, N, K, g, seed=77)
    counts = [9, 30, 16, 0, 12, 40]
    seg_w = [2, -1, 0, -1, 2, -1]
    R = sum(counts)
    x = _w((R, K), seed=3, scale=1.0)
    off = _offsets(counts)
    se = torch.tensor(seg_w, dtype=torch.int32, device="cuda")
    y = w4_gemm(x, packed, N, g, off, hint=hint, seg_expert=se)
    o = off.cpu().tolist()
    ref = torch.zeros(R, N, device="cuda")
    for i, w in enumerate(seg_w):
        if w >= 0 and counts[i]:
            ref[o[i]:o[i + 1]] = x[o[i]:o[i + 1]].float() @ deq[w].T
    _assert_close(y, ref)
    for i, w in enumerate(seg_w):
        if w < 0:
            assert torch.all(y[o[i]:o[i + 1]] == 0), "a hole's output rows were written"


def test_w4_gemm_many_experts_int64_offsets():
    rng = np.random.default_rng(0)
    E = 64
    counts = rng.zipf(1.5, E).clip(0, 400)
    counts[::7] = 0
    N, K, g = 256, 1024, 64
    packed, deq = _expert_setup(E, N, K, g, seed=5)
    R = int(counts.sum())
    x = _w((R, K), seed=9, scale=1.0)
    off = _offsets(counts, torch.int64)
    y = w4_gemm(x, packed, N, g, off)
    _assert_close(y, _ref_plain(x, deq, off))


@pytest.mark.parametrize("counts,hint", [([200, 0, 64, 9], 0), ([3, 16, 40, 64], 64)])
def test_w4_gemm_swiglu(counts, hint):
    E, F, K, g = len(counts), 320, 512, 128
    packed, d1, d3 = _expert_setup(E, F, K, g, seed=3, paired=True)
    R = sum(counts)
    x = _w((R, K), seed=4, scale=1.0)
    off = _offsets(counts)
    h = w4_gemm(x, packed, 2 * F, g, off, epilogue=1, hint=hint)
    gate = _ref_plain(x, d1, off)
    up = _ref_plain(x, d3, off)
    ref = torch.nn.functional.silu(gate) * up
    _assert_close(h, ref)


@pytest.mark.parametrize("epilogue,pad", [(0, 3), (1, 5), (2, 1)])
def test_w4_gemm_unaligned_output_stride(epilogue, pad):
    """Row strides that are not a multiple of 8 elements take the per-element store path."""
    counts = [200, 0, 64, 9]
    E, F, K, g = len(counts), 256, 256, 128
    R = sum(counts)
    x = _w((R, K), seed=6, scale=1.0)
    off = _offsets(counts)
    if epilogue == 1:
        packed, d1, d3 = _expert_setup(E, F, K, g, seed=7, paired=True)
        h = w4_gemm(x, packed, 2 * F, g, off, epilogue=1, pad=pad)
        _assert_close(h, torch.nn.functional.silu(_ref_plain(x, d1, off)) * _ref_plain(x, d3, off))
        return
    packed, deq = _expert_setup(E, F, K, g, seed=7)
    if epilogue == 0:
        _assert_close(w4_gemm(x, packed, F, g, off, pad=pad), _ref_plain(x, deq, off))
        return
    perm = torch.randperm(R + 5, device="cuda")[:R].to(torch.int32)
    scale = torch.rand(R, device="cuda")
    y = w4_gemm(x, packed, F, g, off, epilogue=2, dest=perm, row_scale=scale, out_rows=R + 5, pad=pad)
    ref = torch.zeros(R + 5, F, device="cuda")
    ref[perm.long()] = _ref_plain(x, deq, off) * scale[:, None]
    _assert_close(y, ref)


def test_w4_gemm_scatter():
    counts = [50, 0, 33, 77]
    E, N, K, g = 4, 256, 256, 64
    packed, deq = _expert_setup(E, N, K, g, seed=8)
    R = sum(counts)
    x = _w((R, K), seed=2, scale=1.0)
    off = _offsets(counts)
    perm = torch.randperm(R + 10, device="cuda")[:R].to(torch.int32)
    scale = torch.rand(R, device="cuda")
    y = w4_gemm(x, packed, N, g, off, epilogue=2, dest=perm, row_scale=scale, out_rows=R + 10)
    ref = torch.zeros(R + 10, N, device="cuda")
    ref[perm.long()] = _ref_plain(x, deq, off) * scale[:, None]
    _assert_close(y, ref)


@pytest.mark.parametrize("counts,N,K", [([100, 0, 37, 300], 256, 256), ([7, 1, 64], 200, 128), ([1000, 24], 512, 1024)])
def test_bf16_grouped_gemm(counts, N, K):
    """Dense grouped_gemm (the reference's _C.grouped_gemm) vs a per-expert fp32 loop."""
    E = len(counts)
    w = _w((E, N, K), seed=N)
    R = sum(counts) + 5
    x = _w((R, K), seed=K, scale=1.0)
    off = _offsets(counts, torch.int64)
    y = bf16_gemm(x, w, off)
    ref = _ref_plain(x, w.float(), off)
    _assert_close(y, ref)
    assert torch.all(y[sum(counts):] == 0)   # rows outside every expert are zero (grouped_gemm.cu:24)


def test_reference_grouped_gemm_op():
    from light_moe_b200 import ops
    E, N, K = 4, 128, 256
    w = _w((E, N, K), seed=1)
    x = _w((90, K), seed=2, scale=1.0)
    off = torch.tensor([0, 10, 10, 60, 90], dtype=torch.int64, device="cuda")
    y = ops.grouped_gemm(x, w, off, E)
    _assert_close(y, _ref_plain(x, w.float(), off))


def test_mixtral_grouped_gemms_zipf_full_shape():
    """The Mixtral grouped GEMMs at full shape with a Zipf(1.2) expert load over 8192 rows
    (3516 ... 289 rows per expert, the skewed-GEMM workload): gate/up + SwiGLU, then down,
    checked against fp32 math on the dequantised weights for 48 rows of every segment
    (its first, last and evenly spaced rows), h of the kernel feeding the down reference."""
    E, d, F, g, R = 8, 4096, 14336, 128, 8192
    p = [(i + 1) ** -1.2 for i in range(E)]
    cnt = [int(R * v / sum(p)) for v in p]
    cnt[0] += R - sum(cnt)
    off = np.concatenate([[0], np.cumsum(cnt)]).astype(np.int32)
    gen = torch.Generator(device="cpu").manual_seed(12)
    x = torch.randn(R, d, generator=gen).to(torch.bfloat16).cuda()
    dev = torch.device("cuda")
    q1s, s1s, q3s, s3s, q2s, s2s = [], [], [], [], [], []
    for e in range(E):
        for qs, ss, shape in ((q1s, s1s, (F, d)), (q3s, s3s, (F, d)), (q2s, s2s, (d, F))):
            w = (torch.randn(*shape, generator=gen) * 0.02).to(torch.bfloat16).to(dev)
            q, s = quantize(w, g)
            qs.append(q)
            ss.append(s)
    st = torch.stack
    w13 = prepack(st(q1s), st(s1s), g, st(q3s), st(s3s))
    w2 = prepack(st(q2s), st(s2s), g)
    offsets = torch.from_numpy(off).cuda()
    h = w4_gemm(x, w13, 2 * F, g, offsets, epilogue=1, hint=max(cnt))
    y = w4_gemm(h, w2, d, g, offsets, epilogue=0, hint=max(cnt))
    rows = []
    for e in range(E):
        a, b = int(off[e]), int(off[e + 1])
        rows.extend(np.unique(np.linspace(a, b - 1, 48).astype(np.int64)).tolist())
    idx = torch.tensor(rows, device=dev)
    hs = torch.empty(len(rows), F, device=dev)
    ys = torch.empty(len(rows), d, device=dev)
    for e in range(E):
        sel = [(i, r) for i, r in enumerate(rows) if off[e] <= r < off[e + 1]]
        ii = torch.tensor([i for i, _ in sel], device=dev)
        rr = idx[ii]
        d1 = dequantize(q1s[e], s1s[e], g).float()
        d3 = dequantize(q3s[e], s3s[e], g).float()
        xe = x[rr].float()
        hs[ii] = torch.nn.functional.silu(xe @ d1.T) * (xe @ d3.T)
        del d1, d3
        d2 = dequantize(q2s[e], s2s[e], g).float()
        ys[ii] = h[rr].float() @ d2.T
        del d2
    for got, ref in ((h[idx].float(), hs), (y[idx].float(), ys)):
        err = (got - ref).abs().max().item()
        scale = ref.abs().max().item()
        assert err <= 1e-2 * scale, f"max rel err {err / scale:.3e}"
