"""Seeded input generators shared by the fixture script and the tests.

numpy's PCG64 ``default_rng`` streams are stable across numpy versions, so fixtures store
only outputs and the tests regenerate the inputs from the seed.
"""
from __future__ import annotations

import numpy as np

# (T, d, ffn, E, k, seed) for the SparseMoEBlock fixtures
BLOCK_CASES = [(64, 128, 256, 8, 2, 21), (40, 64, 192, 16, 4, 22), (16, 128, 128, 8, 8, 23)]


def block_inputs(T, d, ffn, E, seed):
    """x ~ N(0,1); router ~ N(0, 0.2); expert weights ~ N(0, 0.05) -- all fp32."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, d), dtype=np.float32)
    gate_w = (rng.standard_normal((E, d), dtype=np.float32) * np.float32(0.2)).astype(np.float32)
    w1 = (rng.standard_normal((E, ffn, d), dtype=np.float32) * np.float32(0.05)).astype(np.float32)
    w3 = (rng.standard_normal((E, ffn, d), dtype=np.float32) * np.float32(0.05)).astype(np.float32)
    w2 = (rng.standard_normal((E, d, ffn), dtype=np.float32) * np.float32(0.05)).astype(np.float32)
    return x, gate_w, w1, w3, w2


def cfg1_inputs(T=512, d=1024, ffn=2816, E=8, seed=0):
    """The CPU-layer workload: x ~ N(0,1), all weights ~ N(0, 0.02), PCG64 seed 0."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, d), dtype=np.float32)
    gate_w = (rng.standard_normal((E, d), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    w1 = (rng.standard_normal((E, ffn, d), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    w3 = (rng.standard_normal((E, ffn, d), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    w2 = (rng.standard_normal((E, d, ffn), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    return x, gate_w, w1, w3, w2
