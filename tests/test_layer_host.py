"""Host-side checks of the layer module that need no GPU: argument validation of
``W4A16MoELayer.forward_host`` and its token-range split (the GPU parity of the call itself
is in test_layer_gpu.py)."""
import pytest
import torch

from light_moe_b200.layer import SMALL_BATCH_TOKENS, W4A16Experts, W4A16MoELayer


def _layer(d=64, E=4, k=2):
    ex = W4A16Experts(torch.empty(0, dtype=torch.uint8), torch.empty(0, dtype=torch.uint8), E, 0, d, 128, 64)
    return W4A16MoELayer(torch.zeros(E, d, dtype=torch.bfloat16), ex, k)


def test_forward_host_rejects_bad_arguments():
    mod = _layer()
    with pytest.raises(ValueError):
        mod.forward_host(torch.zeros(3, 64, dtype=torch.float32))            # not bf16
    with pytest.raises(ValueError):
        mod.forward_host(torch.zeros(3, 64, dtype=torch.bfloat16), out=torch.zeros(3, 32, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        mod.forward_host(torch.zeros(3, 64, dtype=torch.bfloat16), out=torch.zeros(3, 64, dtype=torch.float32))
    with pytest.raises(ValueError):
        mod.forward_host(torch.zeros(4, 64, dtype=torch.bfloat16),
                         out=torch.zeros(64, 4, dtype=torch.bfloat16).t())      # not contiguous


def test_forward_host_empty_batch_needs_no_device():
    mod = _layer()
    out = torch.empty(0, 64, dtype=torch.bfloat16)
    assert mod.forward_host(torch.zeros(0, 64, dtype=torch.bfloat16), out=out) is out


def test_gate_weight_shape_is_checked():
    ex = W4A16Experts(torch.empty(0), torch.empty(0), 4, 0, 64, 128, 64)
    with pytest.raises(ValueError):
        W4A16MoELayer(torch.zeros(4, 32, dtype=torch.bfloat16), ex, 2)


def test_small_batch_threshold_matches_the_router():
    # the host-buffer call keeps every token range above the router's CUDA-core path limit
    import re
    from pathlib import Path
    src = (Path(__file__).resolve().parents[1] / "light_moe_b200" / "csrc" / "router.cu").read_text()
    assert int(re.search(r"constexpr int kSmallTokens = (\d+);", src).group(1)) == SMALL_BATCH_TOKENS


def test_expert_parallel_host_calls_are_one_range():
    # every rank must take the same steps, so the expert-parallel layer refuses to split a
    # host call into token ranges (checked before any device work)
    from light_moe_b200.expert_parallel import ExpertParallelW4A16Layer
    layer = ExpertParallelW4A16Layer.__new__(ExpertParallelW4A16Layer)
    with pytest.raises(ValueError, match="one token range"):
        layer.forward_host_async(torch.zeros(4, 64, dtype=torch.bfloat16), chunks=2)
    with pytest.raises(ValueError, match="one token range"):
        layer.forward_host(torch.zeros(4, 64, dtype=torch.bfloat16), chunks=3)
