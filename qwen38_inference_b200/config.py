"""Hybrid Gated-DeltaNet / gated-GQA model geometry and seeded random-init weights.

The field names follow the checkpoint's ``config.json["text_config"]`` keys that the
reference validates (reference/qwen38_inference.py:4863-4903), so a config dict read
from a real checkpoint maps onto :class:`HybridConfig` one to one.

Presets:

* :func:`qwen38_27b` - the 27B geometry the reference is hard-wired to
  (reference/qwen38_inference.py:4863-4882).
* :func:`tiny` - the CPU-runnable hybrid: hidden 256, 4 layers (3 GDN + 1 attention),
  vocab 1024, fp32 on the CPU restatement.
* :func:`mini` - the same per-head geometry as the 27B model (GDN d=128 with 3 value
  heads per key head, attention d=256 with 6 query heads per KV head, rotary 64) at a
  width and depth the CPU restatement runs in seconds. GPU parity tests use it so that
  every kernel instantiation they exercise is the one the 27B model runs.
"""
from __future__ import annotations

import dataclasses
import math

import torch


@dataclasses.dataclass(frozen=True)
class HybridConfig:
    hidden_size: int
    intermediate_size: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    linear_num_key_heads: int
    linear_num_value_heads: int
    linear_key_head_dim: int
    linear_value_head_dim: int
    linear_conv_kernel_dim: int
    num_hidden_layers: int
    vocab_size: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10_000_000.0
    partial_rotary_factor: float = 0.25
    max_position_embeddings: int = 262_144
    eos_token_id: int = 248_044
    full_attention_interval: int = 4

    # ----- derived sizes (the packed projection widths of reference:4927-4958) -----
    @property
    def layer_types(self) -> list[str]:
        k = self.full_attention_interval
        return ["full_attention" if i % k == k - 1 else "linear_attention" for i in range(self.num_hidden_layers)]

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def q_gate_dim(self) -> int:  # interleaved [q | gate] per query head
        return 2 * self.num_attention_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_key_value_heads * self.head_dim

    @property
    def qkv_dim(self) -> int:  # attention projection rows
        return self.q_gate_dim + 2 * self.kv_dim

    @property
    def attn_out_dim(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def gdn_qk_dim(self) -> int:
        return self.linear_num_key_heads * self.linear_key_head_dim

    @property
    def gdn_v_dim(self) -> int:
        return self.linear_num_value_heads * self.linear_value_head_dim

    @property
    def conv_dim(self) -> int:  # q | k | v channels that go through the causal conv
        return 2 * self.gdn_qk_dim + self.gdn_v_dim

    @property
    def qkvz_dim(self) -> int:
        return self.conv_dim + self.gdn_v_dim

    @property
    def ba_dim(self) -> int:
        return 2 * self.linear_num_value_heads

    def text_config(self) -> dict:
        """The ``text_config`` dict of a checkpoint with this geometry."""
        d = {f.name: getattr(self, f.name) for f in dataclasses.fields(self)}
        d.pop("rope_theta"); d.pop("partial_rotary_factor"); d.pop("full_attention_interval")
        d.update(layer_types=self.layer_types, hidden_act="silu", attn_output_gate=True,
                 attention_bias=False, output_gate_type="swish",
                 rope_parameters={"rope_type": "default", "rope_theta": self.rope_theta,
                                  "partial_rotary_factor": self.partial_rotary_factor})
        return d

    @classmethod
    def from_text_config(cls, c: dict) -> "HybridConfig":
        rp = c.get("rope_parameters", {})
        kw = {f.name: c[f.name] for f in dataclasses.fields(cls) if f.name in c}
        if "rope_theta" in rp:
            kw["rope_theta"] = rp["rope_theta"]
        if "partial_rotary_factor" in rp:
            kw["partial_rotary_factor"] = rp["partial_rotary_factor"]
        eos = c.get("eos_token_id", 248_044)
        kw["eos_token_id"] = eos if isinstance(eos, int) else list(eos)[0]
        return cls(**kw)


def qwen38_27b() -> HybridConfig:
    """The geometry checked at reference/qwen38_inference.py:4863-4882."""
    return HybridConfig(hidden_size=5120, intermediate_size=17408, num_attention_heads=24,
                        num_key_value_heads=4, head_dim=256, linear_num_key_heads=16,
                        linear_num_value_heads=48, linear_key_head_dim=128,
                        linear_value_head_dim=128, linear_conv_kernel_dim=4,
                        num_hidden_layers=64, vocab_size=248320)


def tiny() -> HybridConfig:
    """CPU-runnable hybrid: 3 GDN layers then 1 gated-GQA layer."""
    return HybridConfig(hidden_size=256, intermediate_size=512, num_attention_heads=4,
                        num_key_value_heads=2, head_dim=64, linear_num_key_heads=4,
                        linear_num_value_heads=4, linear_key_head_dim=64,
                        linear_value_head_dim=64, linear_conv_kernel_dim=4,
                        num_hidden_layers=4, vocab_size=1024, partial_rotary_factor=0.25,
                        max_position_embeddings=8192, eos_token_id=7)


def mini(num_layers: int = 4, vocab: int = 2048) -> HybridConfig:
    """27B per-head geometry (GDN 128-d, 3 v-heads per k-head; attention 256-d, GQA 6,
    rotary 64) with a small width so the CPU restatement runs in seconds."""
    return HybridConfig(hidden_size=512, intermediate_size=1024, num_attention_heads=6,
                        num_key_value_heads=1, head_dim=256, linear_num_key_heads=2,
                        linear_num_value_heads=6, linear_key_head_dim=128,
                        linear_value_head_dim=128, linear_conv_kernel_dim=4,
                        num_hidden_layers=num_layers, vocab_size=vocab,
                        max_position_embeddings=65536, eos_token_id=3)


PRESETS = {"27b": qwen38_27b, "tiny": tiny, "mini": mini}


# ---------------------------------------------------------------------------------------
# Seeded random-init weights, in the reference's fused layouts (reference:4927-4958):
#   gate_up = [gate; up]                       [2I, H]
#   qkv     = [q|gate interleaved per head; k; v]  [2*nq*d + 2*nkv*d, H]
#   qkvz    = [q; k; v; z]                     [2*Hk*dk + 2*Hv*dv, H]
#   ba      = [b; a]                           [2*Hv, H]
#   conv    = conv1d.weight[:, 0, :]           [conv_dim, width]
# ---------------------------------------------------------------------------------------

def weight_shapes(cfg: HybridConfig) -> dict:
    """Name -> (shape, dtype-kind) for every tensor, in a fixed order."""
    H = cfg.hidden_size
    out = {"embedding": ((cfg.vocab_size, H), "w"), "final_norm": ((H,), "w"),
           "lm_head": ((cfg.vocab_size, H), "w")}
    for i, kind in enumerate(cfg.layer_types):
        p = f"layers.{i}."
        out[p + "input_norm"] = ((H,), "w")
        out[p + "post_norm"] = ((H,), "w")
        out[p + "gate_up"] = ((2 * cfg.intermediate_size, H), "w")
        out[p + "down"] = ((H, cfg.intermediate_size), "w")
        if kind == "full_attention":
            out[p + "qkv"] = ((cfg.qkv_dim, H), "w")
            out[p + "out"] = ((H, cfg.attn_out_dim), "w")
            out[p + "q_norm"] = ((cfg.head_dim,), "w")
            out[p + "k_norm"] = ((cfg.head_dim,), "w")
        else:
            out[p + "qkvz"] = ((cfg.qkvz_dim, H), "w")
            out[p + "ba"] = ((cfg.ba_dim, H), "w")
            out[p + "conv"] = ((cfg.conv_dim, cfg.linear_conv_kernel_dim), "w")
            out[p + "A_log"] = ((cfg.linear_num_value_heads,), "f32")
            out[p + "dt_bias"] = ((cfg.linear_num_value_heads,), "w")
            out[p + "norm"] = ((cfg.linear_value_head_dim,), "w")
            out[p + "out"] = ((H, cfg.gdn_v_dim), "w")
    return out


def random_weights(cfg: HybridConfig, seed: int = 0, *, dtype=torch.bfloat16, device="cpu",
                   std: float = 0.02, norm_mode: str = "random", shard=None) -> dict:
    """Every tensor i.i.d. N(0, std) from ``seed`` (one generator stream per tensor, so a
    tensor's values do not depend on the device or on the other tensors).

    ``norm_mode="unit"`` sets every Gemma norm weight to 0 (gain 1) and the plain gated
    norm weight to 1, the sensitivity variant of the synthetic-input plan.
    Returns a flat dict ``name -> tensor`` (see :func:`weight_shapes`). ``A_log`` is fp32.
    ``shard(name, tensor) -> tensor``, when given, is applied to each full tensor right after
    it is drawn (tensor parallelism keeps only its rank's slice, so at most one full tensor
    is alive at a time and every rank's slices agree with the unsharded weights).
    """
    device = torch.device(device)
    out = {}
    for idx, (name, (shape, kind)) in enumerate(weight_shapes(cfg).items()):
        gen = torch.Generator(device=device).manual_seed(seed * 1_000_003 + idx)
        t = torch.empty(shape, dtype=torch.float32, device=device)
        t.normal_(0.0, std, generator=gen)
        if norm_mode == "unit":
            if name.endswith(("input_norm", "post_norm", "q_norm", "k_norm")) or name == "final_norm":
                t.zero_()
            elif name.endswith(".norm"):
                t.fill_(1.0)
        t = t if kind == "f32" else t.to(dtype)
        out[name] = shard(name, t) if shard is not None else t
    return out


def nested_layers(flat: dict, cfg: HybridConfig) -> tuple[list[dict], dict]:
    """Split a flat weight dict into the reference's ``layers[i]`` dicts and the globals."""
    layers = [dict() for _ in range(cfg.num_hidden_layers)]
    glob = {}
    for name, t in flat.items():
        if name.startswith("layers."):
            _, i, key = name.split(".", 2)
            layers[int(i)][key] = t
        else:
            glob[name] = t
    return layers, glob


def rope_table(cfg: HybridConfig, max_context: int, device) -> torch.Tensor:
    """``[max_context, rotary_dim]`` fp32 ``[cos | sin]`` table, built with the same torch
    ops as reference/qwen38_inference.py:4904-4909 on ``device``."""
    rd = cfg.rotary_dim
    inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, rd, 2, dtype=torch.float32, device=device) / rd))
    positions = torch.arange(max_context, dtype=torch.float32, device=device)
    freqs = torch.einsum("i,j->ij", positions, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1)


def param_count(cfg: HybridConfig, include_embedding: bool = False) -> int:
    n = 0
    for name, (shape, _) in weight_shapes(cfg).items():
        if name == "embedding" and not include_embedding:
            continue
        n += math.prod(shape)
    return n
