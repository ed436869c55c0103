"""CPU tests: pin the oracle against the reference's own outputs and known answers.

The fixtures under tests/golden/ were produced by running light-moe's PyTorch reference
(tests/golden/make_golden.py).  These tests need no GPU.
"""
import glob
import math
import os

import numpy as np
import pytest

import oracle
from inputs import BLOCK_CASES, block_inputs, cfg1_inputs

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


# ----------------------------------------------------------------------------- conversions
def test_bf16_conversion_matches_round_to_nearest_even():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(100000).astype(np.float32) * 10.0 ** rng.integers(-40, 38, 100000),
                        np.array([0.0, -0.0, 1.0, np.inf, -np.inf, 3.0e38, 1e-45], np.float32)]).astype(np.float32)
    got = oracle.f32_to_bf16_bits(x)
    # independent construction: round half to even on the upper 16 bits via float64 arithmetic
    u = x.view(np.uint32).astype(np.uint64)
    lower = u & 0xFFFF
    upper = u >> 16
    round_up = (lower > 0x8000) | ((lower == 0x8000) & ((upper & 1) == 1))
    want = (upper + round_up).astype(np.uint16)
    assert np.array_equal(got, want)


def test_f16_conversion_matches_numpy():
    rng = np.random.default_rng(1)
    x = np.concatenate([
        rng.standard_normal(200000).astype(np.float32) * 10.0 ** rng.integers(-9, 6, 200000).astype(np.float32),
        np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e6, -1e6, 2.0 ** -24, 2.0 ** -25, 2.0 ** -25 * 1.0001,
                  2.0 ** -14, 2.0 ** -14 * (1 - 2.0 ** -12), np.inf], np.float32)]).astype(np.float32)
    got = oracle.f32_to_f16_bits(x)
    want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)
    back = oracle.f16_bits_to_f32(got)
    assert np.array_equal(back, want.view(np.float16).astype(np.float32))


def test_own_exp_within_two_ulp():
    x = np.linspace(-103.0, 0.0, 2_000_001).astype(np.float32)
    x = np.concatenate([x, -np.abs(np.random.default_rng(2).standard_normal(200000).astype(np.float32)) * 5])
    got = oracle.ref_expf(x).astype(np.float64)
    want = np.exp(x.astype(np.float64))
    normal = want >= 2.0 ** -126
    ulp = np.spacing(want[normal].astype(np.float32)).astype(np.float64)
    err = np.abs(got[normal] - want[normal]) / ulp
    assert err.max() <= 2.0, err.max()
    # subnormal range: absolute error below two subnormal units
    sub = ~normal
    assert np.all(np.abs(got[sub] - want[sub]) <= 2.0 * 2.0 ** -149)
    assert oracle.ref_expf(np.array([0.0], np.float32))[0] == 1.0
    assert oracle.ref_expf(np.array([-200.0], np.float32))[0] == 0.0


# ----------------------------------------------------------------------------- routing
@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "routing_*.npz"))))
def test_routing_matches_reference(path):
    z = np.load(path)
    T, E = z["logits"].shape
    k = z["ids"].shape[1]
    ids, w = oracle.route(z["logits"], k)
    assert np.array_equal(ids, z["ids"]), "expert ids differ from light-moe top_k_routing"
    np.testing.assert_allclose(w, z["weights"], rtol=2e-6, atol=1e-7)
    # reference test_ops.py:116-127 -- weights sum to one
    np.testing.assert_allclose(w.sum(1), np.ones(T), atol=1e-5)
    counts, offsets, _ = oracle.counts_offsets(ids, E)
    assert np.array_equal(counts.astype(np.int64), z["counts"])
    assert offsets[0] == 0 and offsets[-1] == T * k


def test_routing_ties_go_to_lower_expert_id():
    # uniform logits: every expert ties -> ids 0..k-1 (csrc/fused_moe_ops.cu:106-118)
    lg = np.zeros((3, 64), np.float32)
    ids, w = oracle.route(lg, 6)
    assert np.array_equal(ids, np.tile(np.arange(6, dtype=np.int32), (3, 1)))
    np.testing.assert_allclose(w, np.full((3, 6), 1 / 6, np.float32), rtol=1e-6)
    # planted tie between experts 5 and 2 at the top, and 7 / 3 for the second slot
    lg = np.full((1, 8), -1.0, np.float32)
    lg[0, 5] = lg[0, 2] = 2.0
    ids, _ = oracle.route(lg, 2)
    assert ids.tolist() == [[2, 5]]
    lg = np.full((1, 8), -1.0, np.float32)
    lg[0, 6] = 3.0
    lg[0, 7] = lg[0, 3] = 1.0
    ids, _ = oracle.route(lg, 2)
    assert ids.tolist() == [[6, 3]]


def test_routing_degenerate_shapes():
    ids, w = oracle.route(np.zeros((0, 8), np.float32), 2)
    assert ids.shape == (0, 2) and w.shape == (0, 2)
    ids, w = oracle.route(np.array([[0.5, -1.0, 4.0]], np.float32), 3)
    assert ids.tolist() == [[2, 0, 1]]
    np.testing.assert_allclose(w.sum(), 1.0, rtol=1e-6)
    with pytest.raises(ValueError):
        oracle.route(np.zeros((2, 4), np.float32), 5)


# ----------------------------------------------------------------------------- permute
@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "permute_*.npz"))))
def test_permute_matches_reference(path):
    z = np.load(path)
    B, S, k = z["ids"].shape
    E = z["offsets"].shape[0] - 1
    ids = z["ids"].reshape(B * S, k)
    counts, offsets, sidx = oracle.counts_offsets(ids, E)
    assert np.array_equal(offsets.astype(np.int64), z["offsets"])
    # same per-expert segments (reference argsort is unstable -> compare as sorted lists)
    ref_sidx = z["sorted_idx"]
    for e in range(E):
        a, b = offsets[e], offsets[e + 1]
        assert np.array_equal(np.sort(sidx[a:b]), np.sort(ref_sidx[a:b]))
        # stable order inside each segment
        assert np.all(np.diff(sidx[a:b]) > 0)
    # gather rows in the oracle's order: same multiset of rows per segment as the reference
    hid = z["hidden"].reshape(B * S, -1)
    perm = hid[sidx // k]
    for e in range(E):
        a, b = offsets[e], offsets[e + 1]
        ra = perm[a:b][np.lexsort(perm[a:b].T)]
        rb = z["permuted"][a:b][np.lexsort(z["permuted"][a:b].T)]
        assert np.array_equal(ra, rb)
    # unpermute + weighted combine (grouped_gemm.py:250-279) reproduces the reference
    rw = z["rw"].reshape(B * S, k)
    out = np.zeros_like(hid)
    for r in range(B * S * k):
        f = sidx[r]
        out[f // k] += perm[r] * rw[f // k, f % k]
    np.testing.assert_allclose(out, z["unpermuted"].reshape(B * S, -1), rtol=1e-6, atol=1e-6)


# ----------------------------------------------------------------------------- layer
@pytest.mark.parametrize("case", BLOCK_CASES)
def test_block_forward_matches_reference(case):
    T, d, ffn, E, k, seed = case
    z = np.load(os.path.join(GOLDEN, f"block_T{T}_d{d}_f{ffn}_E{E}_k{k}.npz"))
    x, gate_w, w1, w3, w2 = block_inputs(T, d, ffn, E, seed)
    # routing: the oracle reproduces the reference ids on these inputs
    y, ids, w = oracle.moe_layer_ref(x, gate_w, w1, w3, w2, k)
    assert np.array_equal(ids, z["ids"])
    np.testing.assert_allclose(w, z["weights"], rtol=1e-5, atol=1e-7)
    scale = np.abs(z["y"]).max()
    assert np.abs(y - z["y"]).max() <= 1e-5 * scale
    assert np.abs(y - z["y_fast"]).max() <= 1e-5 * scale
    counts, _, _ = oracle.counts_offsets(ids, E)
    assert np.array_equal(counts.astype(np.int64), z["counts"])


def test_cpu_layer_workload_matches_reference():
    z = np.load(os.path.join(GOLDEN, "block_cfg1_summary.npz"))
    x, gate_w, w1, w3, w2 = cfg1_inputs()
    y, ids, w = oracle.moe_layer_ref(x, gate_w, w1, w3, w2, 2)
    assert np.array_equal(ids, z["ids"])
    np.testing.assert_allclose(w, z["weights"], rtol=1e-5, atol=1e-7)
    scale = np.abs(z["y_rows"]).max()
    assert np.abs(y[:16] - z["y_rows"]).max() <= 1e-5 * scale
    norms = np.linalg.norm(y.astype(np.float64), axis=1)
    np.testing.assert_allclose(norms, z["y_row_norms"], rtol=1e-5)
    assert math.isclose(float(np.abs(y.astype(np.float64)).sum()), float(z["y_abs_sum"]), rel_tol=1e-5)


# ----------------------------------------------------------------------------- int4 format
def test_quantize_known_answers():
    g = 8
    # max |w| = 7 -> s = 1 exactly; w/s rounds half to even
    w = np.array([[7.0, -7.0, 2.5, 3.5, -2.5, 0.49, -0.5, 1.5]], np.float32)
    q, s = oracle.quantize_w4(w, g)
    assert oracle.f16_bits_to_f32(s).tolist() == [[1.0]]
    vals = [7, -7, 2, 4, -2, 0, 0, 2]
    want = [((vals[2 * i] + 8) & 15) | (((vals[2 * i + 1] + 8) & 15) << 4) for i in range(4)]
    assert q.tolist() == [want]
    # all-zero group: scale 0, every nibble encodes q = 0 (0x88)
    q0, s0 = oracle.quantize_w4(np.zeros((2, 16), np.float32), 8)
    assert np.all(q0 == 0x88) and np.all(s0 == 0)
    deq = oracle.bf16_bits_to_f32(oracle.dequantize_w4(q0, s0, 8))
    assert np.all(deq == 0)
    # dequantised values: q * s rounded once to bf16
    deq = oracle.bf16_bits_to_f32(oracle.dequantize_w4(q, s, g))
    assert deq.tolist() == [[7.0, -7.0, 2.0, 4.0, -2.0, 0.0, 0.0, 2.0]]


def test_quantize_roundtrip_error_bound():
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((3, 64, 256)) * 0.02).astype(np.float32)
    for g in (64, 128):
        q, s = oracle.quantize_w4(w, g)
        assert q.shape == (3, 64, 128) and s.shape == (3, 64, 256 // g)
        deq = oracle.bf16_bits_to_f32(oracle.dequantize_w4(q, s, g))
        sf = np.repeat(oracle.f16_bits_to_f32(s), g, axis=-1)
        # |w - q s| <= s/2 (fp16 scale rounding widens this by < 1 part in 2^10), then bf16 rounding
        bound = sf * (0.5 + 2.0 ** -9) + np.abs(deq) * 2.0 ** -8
        assert np.all(np.abs(deq - w) <= bound)
        # nibbles are never -8 for symmetric max/7 scaling
        lo, hi = (q & 15).astype(np.int32) - 8, (q >> 4).astype(np.int32) - 8
        assert lo.min() >= -7 and hi.min() >= -7 and lo.max() <= 7 and hi.max() <= 7


def test_quantize_rejects_bad_shapes():
    with pytest.raises(ValueError):
        oracle.quantize_w4(np.zeros((2, 10), np.float32), 4)
