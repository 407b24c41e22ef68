"""Checkpoint directories in the reference's layout (REF:4911-4963).

``load_weights`` reads ``model.safetensors.index.json`` + shards with the tensor names of
reference/qwen38_inference.py:4927-4958 and returns the flat weight dict of
:func:`qwen38_inference_b200.config.weight_shapes` (fused ``gate_up``, ``qkv``, ``qkvz``,
``ba``; ``conv`` as ``[C, W]``), moved to ``device``. ``write_checkpoint`` writes a synthetic
directory in the same layout (config.json with ``text_config``, generation_config.json,
index + one shard), which the reference's own loader accepts for the 27B geometry.
"""
from __future__ import annotations

import json
from pathlib import Path

import torch

from .config import HybridConfig

PREFIX = "model.language_model."


def _names(cfg: HybridConfig):
    """flat name -> list of (checkpoint tensor name, shape) concatenated along dim 0."""
    H = cfg.hidden_size
    out = {"embedding": [(PREFIX + "embed_tokens.weight", (cfg.vocab_size, H))],
           "final_norm": [(PREFIX + "norm.weight", (H,))],
           "lm_head": [("lm_head.weight", (cfg.vocab_size, H))]}
    for i, kind in enumerate(cfg.layer_types):
        p = PREFIX + f"layers.{i}."
        f = f"layers.{i}."
        out[f + "input_norm"] = [(p + "input_layernorm.weight", (H,))]
        out[f + "post_norm"] = [(p + "post_attention_layernorm.weight", (H,))]
        out[f + "down"] = [(p + "mlp.down_proj.weight", (H, cfg.intermediate_size))]
        out[f + "gate_up"] = [(p + "mlp.gate_proj.weight", (cfg.intermediate_size, H)),
                              (p + "mlp.up_proj.weight", (cfg.intermediate_size, H))]
        if kind == "full_attention":
            a = p + "self_attn."
            out[f + "qkv"] = [(a + "q_proj.weight", (cfg.q_gate_dim, H)), (a + "k_proj.weight", (cfg.kv_dim, H)),
                              (a + "v_proj.weight", (cfg.kv_dim, H))]
            out[f + "out"] = [(a + "o_proj.weight", (H, cfg.attn_out_dim))]
            out[f + "q_norm"] = [(a + "q_norm.weight", (cfg.head_dim,))]
            out[f + "k_norm"] = [(a + "k_norm.weight", (cfg.head_dim,))]
        else:
            a = p + "linear_attn."
            out[f + "qkvz"] = [(a + "in_proj_qkv.weight", (cfg.conv_dim, H)), (a + "in_proj_z.weight", (cfg.gdn_v_dim, H))]
            out[f + "ba"] = [(a + "in_proj_b.weight", (cfg.linear_num_value_heads, H)),
                             (a + "in_proj_a.weight", (cfg.linear_num_value_heads, H))]
            out[f + "conv"] = [(a + "conv1d.weight", (cfg.conv_dim, 1, cfg.linear_conv_kernel_dim))]
            out[f + "A_log"] = [(a + "A_log", (cfg.linear_num_value_heads,))]
            out[f + "dt_bias"] = [(a + "dt_bias", (cfg.linear_num_value_heads,))]
            out[f + "norm"] = [(a + "norm.weight", (cfg.linear_value_head_dim,))]
            out[f + "out"] = [(a + "out_proj.weight", (H, cfg.gdn_v_dim))]
    return out


# fused checkpoint tensors accepted in place of a pair of split ones (REF:4944-4953); the
# fused name is preferred when the index holds it, as in REF
FUSED = {"in_proj_qkv.weight": "in_proj_qkvz.weight", "in_proj_z.weight": "in_proj_qkvz.weight",
         "in_proj_b.weight": "in_proj_ba.weight", "in_proj_a.weight": "in_proj_ba.weight"}
ACCEPTED_DTYPES = (torch.bfloat16, torch.float32, torch.float16)


def validate_text_config(c: dict) -> None:
    """The configuration checks of REF:4872-4882 and 4900-4903 that do not pin the 27B
    sizes: the activation, the attention output gate, no bias, the swish gate of the GDN
    norm, unquantized weights, the hybrid layer pattern and the default partial RoPE."""
    if c.get("attention_bias") or c.get("hidden_act") != "silu" or not c.get("attn_output_gate"):
        raise ValueError("Unsupported attention/activation configuration")
    if c.get("output_gate_type", "swish") != "swish" or c.get("quantization_config"):
        raise ValueError("Only unquantized weights with the swish output gate are supported")
    n = c.get("num_hidden_layers")
    interval = c.get("full_attention_interval", 4)
    if c.get("layer_types") is not None and c["layer_types"] != [
            "full_attention" if i % interval == interval - 1 else "linear_attention" for i in range(n)]:
        raise ValueError("Unexpected hybrid attention layout")
    rp = c.get("rope_parameters", {})
    if rp.get("rope_type", "default") != "default":
        raise ValueError("Unsupported rotary embedding configuration")


def load_weights(path, cfg: HybridConfig, device, shard=None) -> dict:
    """Read a checkpoint directory of REF's layout into the flat weight dict (REF:4911-4963):
    every tensor of ``_names(cfg)`` with its shape checked, gate/up, q/k/v and b/a concatenated
    along dim 0, the GDN input projections from their fused form when the index has it.
    Raises ValueError, as REF does, for a missing tensor, a wrong shape, a quantized or other
    unsupported dtype (REF:4922-4923) and any language-model tensor the model does not
    consume other than the MTP head's (REF:4960-4962). ``shard(name, tensor) -> tensor``
    keeps a tensor-parallel rank's slice of each tensor."""
    from safetensors import safe_open
    path = Path(path)
    index = json.loads((path / "model.safetensors.index.json").read_text())["weight_map"]
    loaded = set()

    def read(tname, shape):
        if tname not in index:
            raise ValueError(f"Missing weight: {tname}")
        with safe_open(path / index[tname], framework="pt", device="cpu") as f:
            t = f.get_tensor(tname)
        if tuple(t.shape) != tuple(shape):
            raise ValueError(f"Wrong shape for {tname}: {tuple(t.shape)}, expected {tuple(shape)}")
        if t.dtype not in ACCEPTED_DTYPES:
            raise ValueError(f"Quantized/unsupported weight: {tname} ({t.dtype})")
        loaded.add(tname)
        return t

    flat = {}
    for name, parts in _names(cfg).items():
        base = parts[0][0].rsplit(".", 2)[0] + "."
        fused = FUSED.get(parts[0][0][len(base):]) if len(parts) > 1 else None
        if fused is not None and base + fused in index:
            rows = sum(shape[0] for _, shape in parts)
            t = read(base + fused, (rows,) + tuple(parts[0][1][1:]))
        else:
            ts = [read(tname, shape) for tname, shape in parts]
            t = torch.cat(ts) if len(ts) > 1 else ts[0]
        if name.endswith(".conv"):
            t = t.reshape(t.shape[0], -1)
        t = t.to(device=device, dtype=torch.float32 if name.endswith("A_log") else torch.bfloat16)
        flat[name] = shard(name, t) if shard is not None else t
    unexpected = [n for n in index if n.startswith(PREFIX) and n not in loaded and ".mtp." not in n]
    if unexpected:
        raise ValueError(f"Unconsumed language-model weights: {unexpected[:8]}")
    return flat


def write_checkpoint(path, cfg: HybridConfig, flat: dict, eos_token_id=None) -> Path:
    """Write ``flat`` (config.weight_shapes layout) as a checkpoint directory of REF's layout."""
    from safetensors.torch import save_file
    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    tensors = {}
    for name, parts in _names(cfg).items():
        t = flat[name].detach().cpu()
        if name.endswith(".conv"):
            t = t.reshape(t.shape[0], 1, -1)
        off = 0
        for tname, shape in parts:
            n = shape[0]
            tensors[tname] = t[off:off + n].clone().contiguous() if len(parts) > 1 else t.contiguous()
            off += n
    shard = "model-00001-of-00001.safetensors"
    save_file(tensors, str(path / shard))
    (path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {k: shard for k in tensors}}))
    (path / "config.json").write_text(json.dumps({"text_config": cfg.text_config()}, indent=1))
    (path / "generation_config.json").write_text(json.dumps({"eos_token_id": eos_token_id or cfg.eos_token_id}))
    return path
