"""CPU oracle for the MoE-layer hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may
import this package.  The product (``light_moe_b200``) never does: it fails loudly when its
CUDA library is missing instead of falling back to anything here.

Contents
--------
* ``lmoe_oracle.c`` (built to ``_build/liblmoe_oracle.so`` by ``Makefile``): bit-exact C
  restatement of routing (softmax / top-k / renormalise), counts / offsets / stable
  permutation, and the int4 quantise / dequantise format.  Loaded here through ctypes.
* ``layer.py``: numpy fp32 restatement of light-moe's ``SparseMoEBlock.forward``
  (python/light_moe/model/moe_block.py:119-169) and of its expert MLP
  (moe_block.py:50-60, swiglu at python/light_moe/ops/activation.py:30-50).

Pinning: ``tests/golden/make_golden.py`` imports the reference package in the development
container and records its outputs as fixtures; ``tests/test_oracle.py`` checks this oracle
against them.
"""
from .core import (  # noqa: F401
    build_oracle,
    load,
    f32_to_bf16_bits,
    bf16_bits_to_f32,
    f32_to_f16_bits,
    f16_bits_to_f32,
    ref_expf,
    route,
    softmax_probs,
    counts_offsets,
    quantize_w4,
    dequantize_w4,
)
from .layer import (  # noqa: F401
    gate_logits_f64,
    moe_layer_ref,
    expert_mlp_ref,
    reference_block_forward,
)
