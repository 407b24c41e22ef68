"""Checkpoint directories in the reference's layout (REF:4911-4963): write -> load round trip,
the fused GDN input projections, and the reference loader's rejections. CPU only.

The last test runs the reference's own ``_load_weights`` over the index this repository
writes for the 27B geometry, with the tensors replaced by shape-only (meta) stand-ins, so the
tensor names and shapes are checked against the reference loader itself without 54 GB of
data. It is skipped where the reference checkout is not present.
"""
import json
import sys
from pathlib import Path

import pytest
import torch

from qwen38_inference_b200.checkpoint import PREFIX, _names, load_weights, write_checkpoint
from qwen38_inference_b200.config import mini, qwen38_27b, random_weights, weight_shapes
from qwen38_inference_b200.model import load_checkpoint_config

REF_ROOT = Path("/root/reference")


@pytest.fixture
def ckpt(tmp_path):
    cfg = mini(num_layers=4, vocab=64)
    w = random_weights(cfg, seed=5)
    write_checkpoint(tmp_path, cfg, w)
    return tmp_path, cfg, w


def _rewrite(path, edit):
    """Load every tensor of the checkpoint, let ``edit(tensors)`` change the dict, write it
    back as one shard with a fresh index."""
    from safetensors.torch import load_file, save_file
    shard = path / "model-00001-of-00001.safetensors"
    tensors = load_file(str(shard))
    edit(tensors)
    save_file(tensors, str(shard))
    (path / "model.safetensors.index.json").write_text(
        json.dumps({"weight_map": {k: shard.name for k in tensors}}))


def test_round_trip_bit_exact(ckpt):
    path, cfg, w = ckpt
    assert load_checkpoint_config(path) == cfg
    got = load_weights(path, cfg, "cpu")
    assert set(got) == set(weight_shapes(cfg))
    for k, v in w.items():
        assert got[k].dtype == v.dtype and torch.equal(got[k], v), k


def test_fused_gdn_projections(ckpt):
    """in_proj_qkvz / in_proj_ba in place of the split tensors (REF:4944-4953) load to the same
    weights; a fused tensor of the wrong shape is rejected."""
    path, cfg, w = ckpt

    def fuse(t):
        for i, kind in enumerate(cfg.layer_types):
            if kind == "full_attention":
                continue
            a = PREFIX + f"layers.{i}.linear_attn."
            t[a + "in_proj_qkvz.weight"] = torch.cat([t.pop(a + "in_proj_qkv.weight"), t.pop(a + "in_proj_z.weight")])
            t[a + "in_proj_ba.weight"] = torch.cat([t.pop(a + "in_proj_b.weight"), t.pop(a + "in_proj_a.weight")])
    _rewrite(path, fuse)
    got = load_weights(path, cfg, "cpu")
    for k, v in w.items():
        assert torch.equal(got[k], v), k

    def truncate(t):
        a = PREFIX + "layers.0.linear_attn.in_proj_ba.weight"
        t[a] = t[a][:-1].clone()
    _rewrite(path, truncate)
    with pytest.raises(ValueError, match="Wrong shape"):
        load_weights(path, cfg, "cpu")


def test_rejections(ckpt):
    path, cfg, _ = ckpt
    name = PREFIX + "layers.0.mlp.down_proj.weight"

    _rewrite(path, lambda t: t.__setitem__(name, t[name].to(torch.int8)))
    with pytest.raises(ValueError, match="Quantized/unsupported"):
        load_weights(path, cfg, "cpu")
    _rewrite(path, lambda t: t.__setitem__(name, t[name].to(torch.bfloat16)))
    load_weights(path, cfg, "cpu")

    _rewrite(path, lambda t: t.__setitem__(PREFIX + "layers.1.mlp.extra.weight", torch.zeros(2)))
    with pytest.raises(ValueError, match="Unconsumed"):
        load_weights(path, cfg, "cpu")
    _rewrite(path, lambda t: (t.pop(PREFIX + "layers.1.mlp.extra.weight"),
                              t.__setitem__(PREFIX + "mtp.layers.0.extra.weight", torch.zeros(2))))
    load_weights(path, cfg, "cpu")  # the MTP head's tensors are not the model's (REF:4960)

    _rewrite(path, lambda t: t.pop(name))
    with pytest.raises(ValueError, match="Missing weight"):
        load_weights(path, cfg, "cpu")

    conf = json.loads((path / "config.json").read_text())
    for key, bad in (("quantization_config", {"quant_method": "fp8"}), ("hidden_act", "gelu"),
                     ("attn_output_gate", False), ("output_gate_type", "sigmoid"),
                     ("layer_types", ["linear_attention"] * cfg.num_hidden_layers)):
        c = json.loads(json.dumps(conf))
        c["text_config"][key] = bad
        (path / "config.json").write_text(json.dumps(c))
        with pytest.raises(ValueError):
            load_checkpoint_config(path)


@pytest.mark.skipif(not (REF_ROOT / "reference" / "qwen38_inference.py").exists(), reason="reference not present")
def test_reference_loader_accepts_the_27b_index(monkeypatch):
    """The reference's ``Qwen38._load_weights`` (REF:4911-4963) reads the names and shapes
    this repository writes for the 27B geometry: every tensor is found with the shape it
    expects, and nothing is left unconsumed."""
    sys.path.insert(0, str(REF_ROOT))
    try:
        import reference.qwen38_inference as R
    except Exception as e:  # pragma: no cover - the import needs triton and safetensors
        pytest.skip(f"reference import failed: {e}")
    cfg = qwen38_27b()
    shapes = {}
    for parts in _names(cfg).values():
        for tname, shape in parts:
            shapes[tname] = shape
    index = {"weight_map": {k: "model-00001-of-00001.safetensors" for k in shapes}}

    class Stub:
        def __init__(self, *a, **k):
            pass

        def __enter__(self):
            return self

        def __exit__(self, *a):
            return False

        def get_tensor(self, name):
            return torch.empty(shapes[name], dtype=torch.bfloat16, device="meta")

    monkeypatch.setattr(R, "safe_open", Stub)
    m = object.__new__(R.Qwen38)
    m.path = Path("/nonexistent")
    m.device, m.dtype = torch.device("meta"), torch.bfloat16
    m.layer_types = cfg.layer_types
    monkeypatch.setattr(Path, "read_text", lambda self, *a, **k: json.dumps(index))
    m._load_weights()
    assert set(m.loaded_weight_names) == set(shapes)
    assert m.lm_head.shape == (cfg.vocab_size, cfg.hidden_size)
    assert m.layers[0]["qkvz"].shape == (cfg.qkvz_dim, cfg.hidden_size)
    assert m.layers[3]["qkv"].shape == (cfg.qkv_dim, cfg.hidden_size)
