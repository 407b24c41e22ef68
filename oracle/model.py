"""CPU restatement of ``Qwen38`` cache bookkeeping and ``forward_step`` (TEST INFRASTRUCTURE ONLY).

Follows reference/qwen38_inference.py ("REF") in this order: ``_token_batch``
(REF:4821-4841) -> validation and metadata (REF:5013-5044) -> embedding -> per layer
(norm, attention or GDN mixer, MLP; REF:5047-5092) -> final norm, last-row select,
lm_head, ``.float()`` (REF:5093-5096) -> commit lengths (REF:5097-5098).
"""
from __future__ import annotations

import dataclasses
import math

import torch

from . import ops

PAGE = 64


@dataclasses.dataclass
class HybridCacheCPU:
    """The reference ``HybridCache`` (REF:4786-4818) on the CPU."""
    owner: int
    lengths: list
    capacity: int
    max_context: int
    kv: dict
    conv: dict
    recurrent: dict

    def clone(self):
        return HybridCacheCPU(self.owner, self.lengths.copy(), self.capacity, self.max_context,
                              {i: (k.clone(), v.clone()) for i, (k, v) in self.kv.items()},
                              {i: x.clone() for i, x in self.conv.items()},
                              {i: x.clone() for i, x in self.recurrent.items()})

    def reset(self, request_indices=None):
        """REF:4808-4818: zero lengths, conv and recurrent state; KV rows are left stale."""
        slots = list(range(len(self.lengths))) if request_indices is None else list(request_indices)
        if len(set(slots)) != len(slots) or any(i < 0 or i >= len(self.lengths) for i in slots):
            raise ValueError("Invalid or duplicate cache slots")
        for s in slots:
            self.lengths[s] = 0
            for st in self.conv.values():
                st[s].zero_()
            for st in self.recurrent.values():
                st[s].zero_()


def token_batch(input_ids):
    """REF:4821-4841."""
    if isinstance(input_ids, torch.Tensor):
        if input_ids.ndim not in (1, 2) or input_ids.dtype not in (torch.int32, torch.int64):
            raise ValueError("input_ids must be a 1D or 2D integer tensor")
        input_ids = input_ids.tolist()
    if not isinstance(input_ids, (list, tuple)) or len(input_ids) == 0:
        raise ValueError("input_ids must contain at least one nonempty sequence")
    single = isinstance(input_ids[0], int)
    rows = [input_ids] if single else input_ids
    result = []
    for row in rows:
        if isinstance(row, torch.Tensor):
            if row.ndim != 1 or row.dtype not in (torch.int32, torch.int64):
                raise ValueError("Each request must be a 1D integer sequence")
            row = row.tolist()
        if not isinstance(row, (list, tuple)) or not row:
            raise ValueError("Empty requests and padded tensors are not accepted; pass unpadded lists")
        if any(type(t) is not int for t in row):
            raise ValueError("Token IDs must be integers")
        result.append(list(row))
    return result, single


def metadata(cache_lengths, capacity, slots, lens):
    """REF:5023-5044 as plain Python lists (no device): the bit-exact bookkeeping."""
    prefixes = [cache_lengths[s] for s in slots]
    lengths = [p + n for p, n in zip(prefixes, lens)]
    cu, kv_cu = [0], [0]
    for n, L in zip(lens, lengths):
        cu.append(cu[-1] + n)
        kv_cu.append(kv_cu[-1] + L)
    positions = [p + j for p, n in zip(prefixes, lens) for j in range(n)]
    locations = [PAGE + s * capacity + p + j for s, p, n in zip(slots, prefixes, lens) for j in range(n)]
    pps = capacity // PAGE
    max_pages = math.ceil(max(lengths) / PAGE)
    page_table = [[1 + s * pps + j if j < math.ceil(n / PAGE) else 0 for j in range(max_pages)]
                  for s, n in zip(slots, lengths)]
    return dict(prefixes=prefixes, lengths=lengths, cu=cu, kv_cu=kv_cu, positions=positions,
                locations=locations, page_table=page_table, has_initial=[p > 0 for p in prefixes],
                is_decode=all(n == 1 and p > 0 for n, p in zip(lens, prefixes)))


class OracleModel:
    """CPU forward of the hybrid model. ``dtype`` is the storage dtype: bf16 reproduces the
    27B model's rounding points, fp32 is the tiny configuration's arithmetic."""

    def __init__(self, cfg, weights: dict, *, dtype=torch.bfloat16, max_context=None, gdn_prefill_form="token"):
        """``gdn_prefill_form``: "token" runs prefill GDN as the per-token recurrence (the
        reference's definition, REF:1355-1408 applied per token); "chunked" as the chunked form
        with bf16 operands of oracle/chunked.py (the arithmetic of the prefill kernel, whose
        algorithm the reference's flashinfer chunked kernel shares)."""
        from qwen38_inference_b200.config import nested_layers, rope_table  # pure-Python helpers
        if gdn_prefill_form not in ("token", "chunked"):
            raise ValueError("gdn_prefill_form must be 'token' or 'chunked'")
        self.gdn_prefill_form = gdn_prefill_form
        self.cfg = cfg
        self.dtype = dtype
        self.rnd = ops.bf16 if dtype == torch.bfloat16 else ops.ident
        self.eps = cfg.rms_norm_eps
        self.page_size = PAGE
        self.max_context = cfg.max_position_embeddings if max_context is None else int(max_context)
        self.layer_types = cfg.layer_types
        w = {k: (v.float() if v.dtype == torch.float32 else v.to(dtype)).cpu() for k, v in weights.items()}
        self.layers, g = nested_layers(w, cfg)
        self.embedding, self.final_norm, self.lm_head = g["embedding"], g["final_norm"], g["lm_head"]
        self.rope = rope_table(cfg, self.max_context, "cpu")

    # ------------------------------------------------------------------ cache (REF:4966-5001)
    def new_cache(self, batch_size=1, initial_capacity=256, max_context=None):
        c = self.cfg
        if not isinstance(batch_size, int) or batch_size < 1:
            raise ValueError("batch_size must be a positive integer")
        limit = self.max_context if max_context is None else int(max_context)
        if not 1 <= limit <= self.max_context or initial_capacity < 1:
            raise ValueError("Invalid cache capacity/context limit")
        cap = math.ceil(min(initial_capacity, limit) / PAGE) * PAGE
        kv, conv, rec = {}, {}, {}
        for i, kind in enumerate(self.layer_types):
            if kind == "full_attention":
                shape = (batch_size * cap + PAGE, c.num_key_value_heads, c.head_dim)
                kv[i] = (torch.zeros(shape, dtype=self.dtype), torch.zeros(shape, dtype=self.dtype))
            else:
                conv[i] = torch.zeros(batch_size, c.conv_dim, c.linear_conv_kernel_dim - 1, dtype=self.dtype)
                rec[i] = torch.zeros(batch_size, c.linear_num_value_heads, c.linear_value_head_dim,
                                     c.linear_key_head_dim, dtype=torch.float32)
        return HybridCacheCPU(id(self), [0] * batch_size, cap, limit, kv, conv, rec)

    def _reserve(self, cache, needed):
        if needed > cache.max_context:
            raise ValueError(f"Context limit exceeded: {needed} > {cache.max_context}")
        if needed <= cache.capacity:
            return
        cap = math.ceil(min(cache.max_context, max(needed, cache.capacity * 2)) / PAGE) * PAGE
        new_kv = {}
        for i, pair in cache.kv.items():
            new_pair = []
            for old in pair:
                new = torch.zeros((len(cache.lengths) * cap + PAGE,) + tuple(old.shape[1:]), dtype=old.dtype)
                for s, L in enumerate(cache.lengths):
                    new[PAGE + s * cap:PAGE + s * cap + L] = old[PAGE + s * cache.capacity:PAGE + s * cache.capacity + L]
                new_pair.append(new)
            new_kv[i] = tuple(new_pair)
        cache.kv = new_kv
        cache.capacity = cap

    # ------------------------------------------------------------------ forward (REF:5004-5099)
    @torch.inference_mode()
    def forward_step(self, input_ids, kv_cache, *, request_indices=None, return_all_logits=False, trace=None):
        """REF:5004-5099. ``trace`` (a list) receives the layer loop's state at every half-layer
        boundary as (hidden, residual) pairs, storage-dtype values as fp32: entry 2i is layer
        i's normalized input, entry 2i + 1 the normalized input of its MLP, and the last entry
        the last down projection's output with the residual before the final norm."""
        c, rnd, eps = self.cfg, self.rnd, self.eps
        rows, _ = token_batch(input_ids)
        cache = kv_cache
        if not isinstance(cache, HybridCacheCPU) or cache.owner != id(self):
            raise ValueError("kv_cache must have been created by this model")
        slots = list(range(len(cache.lengths))) if request_indices is None else list(request_indices)
        if len(slots) != len(rows) or len(set(slots)) != len(slots) or any(
                type(s) is not int or s < 0 or s >= len(cache.lengths) for s in slots):
            raise ValueError("request_indices must identify one distinct cache slot per input sequence")
        flat = [t for r in rows for t in r]
        if any(t < 0 or t >= c.vocab_size for t in flat):
            raise ValueError("Token ID outside model vocabulary")
        lens = [len(r) for r in rows]
        self._reserve(cache, max(cache.lengths[s] + n for s, n in zip(slots, lens)))
        md = metadata(cache.lengths, cache.capacity, slots, lens)
        positions = torch.tensor(md["positions"], dtype=torch.int64)
        locations = torch.tensor(md["locations"], dtype=torch.int64)
        starts = [PAGE + s * cache.capacity for s in slots]

        hidden = ops.f32(self.embedding[torch.tensor(flat, dtype=torch.int64)])
        residual = None
        nq, nkv, d = c.num_attention_heads, c.num_key_value_heads, c.head_dim
        H, HV, dk, dv = c.linear_num_key_heads, c.linear_num_value_heads, c.linear_key_head_dim, c.linear_value_head_dim
        for i, (kind, w) in enumerate(zip(self.layer_types, self.layers)):
            if residual is None:
                residual = hidden
                hidden = ops.gemma_rmsnorm(hidden, w["input_norm"], eps, rnd)
            else:
                hidden, residual = ops.gemma_add_rmsnorm(hidden, residual, w["input_norm"], eps, rnd)
            if trace is not None:
                trace.append((hidden.clone(), residual.clone()))
            if kind == "full_attention":
                proj = ops.linear(hidden, w["qkv"], rnd)
                qg, k, v = proj.split([c.q_gate_dim, c.kv_dim, c.kv_dim], dim=-1)
                q, k, gate = ops.qk_norm_rope_gate(qg, k, w["q_norm"], w["k_norm"], self.rope, positions,
                                                   eps, nq, nkv, d, c.rotary_dim, rnd)
                kc, vc = cache.kv[i]
                kc[locations] = k.to(kc.dtype)
                vc[locations] = v.reshape(-1, nkv, d).to(vc.dtype)
                att = ops.paged_attention(q, kc, vc, starts, md["prefixes"], lens, d ** -0.5, rnd)
                out = ops.sigmoid_mul(att.reshape(-1, nq * d), gate.reshape(-1, nq * d), rnd)
                hidden = ops.linear(out, w["out"], rnd)
            else:
                qkvz = ops.linear(hidden, w["qkvz"], rnd)
                ba = ops.linear(hidden, w["ba"], rnd)
                mixed_in, z = qkvz[:, :c.conv_dim], qkvz[:, c.conv_dim:]
                b, a = ba[:, :HV], ba[:, HV:]
                g, beta = ops.gdn_gating(w["A_log"], a, b, w["dt_bias"], rnd)
                if md["is_decode"]:
                    mixed = ops.conv_decode(mixed_in, w["conv"], cache.conv[i], slots, rnd)
                    q = ops.l2norm(mixed[:, :c.gdn_qk_dim].reshape(-1, H, dk))
                    k = ops.l2norm(mixed[:, c.gdn_qk_dim:2 * c.gdn_qk_dim].reshape(-1, H, dk))
                else:
                    mixed = ops.conv_prefill(mixed_in, w["conv"], cache.conv[i], md["cu"], slots,
                                             md["has_initial"], rnd)
                    q = rnd(ops.l2norm(mixed[:, :c.gdn_qk_dim].reshape(-1, H, dk)))
                    k = rnd(ops.l2norm(mixed[:, c.gdn_qk_dim:2 * c.gdn_qk_dim].reshape(-1, H, dk)))
                v = mixed[:, 2 * c.gdn_qk_dim:].reshape(-1, HV, dv)
                o = torch.empty(len(flat), HV, dv)
                rec = cache.recurrent[i]
                for j, s in enumerate(slots):
                    a0, a1 = md["cu"][j], md["cu"][j + 1]
                    if self.gdn_prefill_form == "chunked" and not md["is_decode"]:
                        from .chunked import chunked_gdn
                        o[a0:a1], rec[s] = chunked_gdn(q[a0:a1], k[a0:a1], v[a0:a1], a[a0:a1], b[a0:a1], w["A_log"],
                                                       w["dt_bias"], rec[s], dk ** -0.5, HV // H)
                        continue
                    o[a0:a1], rec[s] = ops.gdn_recurrence(q[a0:a1], k[a0:a1], v[a0:a1], g[a0:a1],
                                                          beta[a0:a1], rec[s], dk ** -0.5, HV // H)
                o = rnd(o)
                y = ops.gated_rmsnorm(o.reshape(-1, dv), w["norm"], z.reshape(-1, dv), eps, rnd)
                hidden = ops.linear(y.reshape(-1, c.gdn_v_dim), w["out"], rnd)
            hidden, residual = ops.gemma_add_rmsnorm(hidden, residual, w["post_norm"], eps, rnd)
            if trace is not None:
                trace.append((hidden.clone(), residual.clone()))
            act = ops.silu_mul(ops.linear(hidden, w["gate_up"], rnd), rnd)
            hidden = ops.linear(act, w["down"], rnd)
        if trace is not None:
            trace.append((hidden.clone(), residual.clone()))
        hidden, residual = ops.gemma_add_rmsnorm(hidden, residual, self.final_norm, eps, rnd)
        if not return_all_logits:
            hidden = hidden[torch.tensor([e - 1 for e in md["cu"][1:]], dtype=torch.int64)]
        logits = ops.linear(hidden, self.lm_head, rnd).float()
        for s, L in zip(slots, md["lengths"]):
            cache.lengths[s] = L
        return logits

    # ------------------------------------------------------------------ generate (REF:5102-5147)
    @torch.inference_mode()
    def generate(self, input_ids, *, max_new_tokens=None, eos_token_ids=None, prefill_chunk_size=512):
        rows, single = token_batch(input_ids)
        eos = {self.cfg.eos_token_id} if eos_token_ids is None else (
            {eos_token_ids} if isinstance(eos_token_ids, int) else set(eos_token_ids))
        output = [[] for _ in rows]
        if max_new_tokens == 0:
            return output[0] if single else output
        cache = self.new_cache(len(rows))
        last = {}
        for off in range(0, max(map(len, rows)), prefill_chunk_size):
            slots = [i for i, r in enumerate(rows) if off < len(r)]
            logits = self.forward_step([rows[i][off:off + prefill_chunk_size] for i in slots], cache,
                                       request_indices=slots)
            for j, s in enumerate(slots):
                last[s] = logits[j]
        active = list(range(len(rows)))
        logits = torch.stack([last[i] for i in active])
        while active:
            toks = logits.argmax(-1).tolist()
            nxt, inp = [], []
            for s, t in zip(active, toks):
                output[s].append(t)
                if t in eos or (max_new_tokens is not None and len(output[s]) >= max_new_tokens):
                    continue
                if cache.lengths[s] >= cache.max_context:
                    raise RuntimeError(f"Request {s} exhausted context without EOS; produced {len(output[s])} tokens")
                nxt.append(s)
                inp.append([t])
            active = nxt
            if active:
                logits = self.forward_step(inp, cache, request_indices=active)
        return output[0] if single else output
