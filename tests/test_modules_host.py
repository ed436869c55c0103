"""Host-side tests of the model-facing modules (no GPU):

* ``loader``: the safetensors container (round trip, interoperability with the
  ``safetensors`` package when it is installed), Mixtral checkpoint discovery and the
  reference's role map w1 -> gate_proj, w3 -> up_proj, w2 -> down_proj
  (python/light_moe/model/loader.py:119-128), and the int4 file's format check;
* ``integration``: reading both light-moe block layouts (SparseMoEBlock's ModuleList of
  experts, SparseMoEBlockFast's grouped projections) and the model-level switch;
* ``router``: the load-balancing loss against the reference's own values (golden fixtures
  recorded from python/light_moe/ops/moe_gate.py:80-122).
"""
import glob
import json
import os

import numpy as np
import pytest
import torch

from light_moe_b200 import integration, loader
from light_moe_b200.router import MoEGate, load_balancing_loss
from model_fixtures import FastBlockLike, SparseBlockLike, make_mixtral_dir

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_safetensors_round_trip(tmp_path):
    g = torch.Generator().manual_seed(0)
    ts = {
        "a.bf16": torch.randn(3, 5, generator=g).to(torch.bfloat16),
        "b.f16": torch.randn(7, generator=g).to(torch.float16),
        "c.f32": torch.randn(2, 2, 2, generator=g),
        "d.u8": torch.randint(0, 256, (9, 4), dtype=torch.uint8, generator=g),
        "e.i64": torch.arange(5, dtype=torch.int64),
        "f.empty": torch.empty(0, 3, dtype=torch.float32),
    }
    p = str(tmp_path / "x.safetensors")
    loader.write_safetensors(p, ts, {"k": 1, "s": "v"})
    with loader.SafetensorsFile(p) as st:
        assert st.metadata == {"k": "1", "s": "v"}
        assert sorted(st.keys()) == sorted(ts)
        for n, t in ts.items():
            got = st.get(n)
            assert got.dtype == t.dtype and got.shape == t.shape
            assert torch.equal(got, t)


def test_safetensors_interoperates_with_the_package(tmp_path):
    st_pkg = pytest.importorskip("safetensors.torch")
    from safetensors import safe_open
    t = {"w": torch.randn(4, 6).to(torch.bfloat16), "q": torch.randint(0, 255, (3, 3), dtype=torch.uint8)}
    ours = str(tmp_path / "ours.safetensors")
    loader.write_safetensors(ours, t, {"format": "x"})
    with safe_open(ours, framework="pt") as f:
        assert f.metadata() == {"format": "x"}
        for n in t:
            assert torch.equal(f.get_tensor(n), t[n])
    theirs = str(tmp_path / "theirs.safetensors")
    st_pkg.save_file(t, theirs, metadata={"a": "b"})
    with loader.SafetensorsFile(theirs) as st:
        assert st.metadata == {"a": "b"}
        for n in t:
            assert torch.equal(st.get(n), t[n])


def test_safetensors_rejects_corrupt_headers(tmp_path):
    p = tmp_path / "bad.safetensors"
    p.write_bytes((1 << 40).to_bytes(8, "little") + b"{}")
    with pytest.raises(ValueError):
        loader.SafetensorsFile(str(p))
    hdr = json.dumps({"x": {"dtype": "F32", "shape": [4], "data_offsets": [0, 1000]}}).encode()
    p.write_bytes(len(hdr).to_bytes(8, "little") + hdr + b"\0" * 16)
    with pytest.raises(ValueError):
        loader.SafetensorsFile(str(p))


def test_mixtral_checkpoint_roles_and_shards(tmp_path):
    cfg, ref = make_mixtral_dir(str(tmp_path / "mx"), L=3, E=4, d=64, F=128)
    c = loader.read_hf_config(str(tmp_path / "mx"))
    assert c == {"hidden_size": 64, "intermediate_size": 128, "num_experts": 4, "top_k": 2, "num_layers": 3}
    assert len(loader.hf_weight_files(str(tmp_path / "mx"))) == 2
    got = dict(loader.iter_hf_moe_layers(str(tmp_path / "mx")))
    assert sorted(got) == [0, 1, 2]
    for li, w in got.items():
        assert torch.equal(w["gate"], ref[li]["gate"])
        # w1 = gate_proj [E, ffn, d], w3 = up_proj [E, ffn, d], w2 = down_proj [E, d, ffn]
        assert w["w1"].shape == (4, 128, 64) and w["w3"].shape == (4, 128, 64) and w["w2"].shape == (4, 64, 128)
        for r in ("w1", "w3", "w2"):
            assert torch.equal(w[r], torch.stack(ref[li][r]))
    assert loader.ROLES == {"w1": "gate_proj", "w3": "up_proj", "w2": "down_proj"}
    only = dict(loader.iter_hf_moe_layers(str(tmp_path / "mx"), layers=[1]))
    assert list(only) == [1]
    with pytest.raises(KeyError):
        dict(loader.iter_hf_moe_layers(str(tmp_path / "mx"), layers=[7]))


def test_mixtral_checkpoint_missing_expert(tmp_path):
    d = str(tmp_path / "mx")
    make_mixtral_dir(d, L=1, E=4, shards=1)
    f = loader.hf_weight_files(d)[0]
    with loader.SafetensorsFile(f) as st:
        ts = {n: st.get(n).clone() for n in st.keys() if ".experts.3.w2." not in n}
    loader.write_safetensors(f, ts)
    with pytest.raises(KeyError):
        dict(loader.iter_hf_moe_layers(d))


def test_int4_file_format_is_checked(tmp_path):
    p = str(tmp_path / "w.safetensors")
    loader.write_safetensors(p, {"x": torch.zeros(2)}, {"format": "something-else"})
    with pytest.raises(ValueError):
        loader.load_w4a16(p, device="cpu")
    loader.write_safetensors(p, {"x": torch.zeros(2)}, {"format": loader.FORMAT, "version": "99"})
    with pytest.raises(ValueError):
        loader.load_w4a16(p, device="cpu")


# ------------------------------------------------------------------------------ block layouts
def test_block_weights_from_both_layouts():
    b = SparseBlockLike()
    w = integration.block_weights(b)
    assert w["top_k"] == 2 and w["aux_loss_coef"] == pytest.approx(0.02) and w["gate_bias"] is None
    assert torch.equal(w["w1"][2], b.experts[2].gate_proj.weight)
    assert torch.equal(w["w3"][1], b.experts[1].up_proj.weight)
    assert torch.equal(w["w2"][3], b.experts[3].down_proj.weight)
    f = FastBlockLike()
    w = integration.block_weights(f)
    assert torch.equal(w["w1"], f.gate_proj.weight) and torch.equal(w["w2"], f.down_proj.weight)
    bad = SparseBlockLike()
    bad.experts[0].up_proj = torch.nn.Linear(64, 128, bias=True)
    with pytest.raises(ValueError):
        integration.block_weights(bad)


def test_enable_w4a16_replaces_every_block(monkeypatch):
    class Layer(torch.nn.Module):
        def __init__(self, fast):
            super().__init__()
            self.moe = FastBlockLike() if fast else SparseBlockLike()
            self.norm = torch.nn.LayerNorm(64)

    model = torch.nn.ModuleList([Layer(False), Layer(True), Layer(False)])
    seen = []

    def fake_convert(block, group_size=128, device=None):
        seen.append((type(block).__name__, group_size))
        return torch.nn.Identity()

    monkeypatch.setattr(integration, "convert_block", fake_convert)
    assert integration.enable_w4a16(model, group_size=64) == 3
    assert [s[0] for s in seen] == ["SparseBlockLike", "FastBlockLike", "SparseBlockLike"]
    assert all(isinstance(l.moe, torch.nn.Identity) for l in model)
    assert all(isinstance(l.norm, torch.nn.LayerNorm) for l in model)


# ------------------------------------------------------------------------------ router module
@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "routing_*.npz"))))
def test_load_balancing_loss_matches_reference(path):
    z = np.load(path)
    T, E = z["probs"].shape
    k = z["ids"].shape[1]
    probs = torch.from_numpy(z["probs"]).view(1, T, E)
    ids = torch.from_numpy(z["ids"].astype(np.int64)).view(1, T, k)
    got = load_balancing_loss(probs, ids, E).item()
    assert got == pytest.approx(float(z["aux_loss"]), rel=1e-6, abs=1e-7)


def test_moe_gate_module_keeps_the_reference_parameters():
    g = MoEGate(64, 8, top_k=2, bias=True)
    assert sorted(dict(g.named_parameters())) == ["gate.bias", "gate.weight"]
    assert g.gate.weight.shape == (8, 64)
    with pytest.raises(ValueError):
        MoEGate(64, 8, routing_type="sigmoid")
