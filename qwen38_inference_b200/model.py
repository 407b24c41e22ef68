"""Drop-in ``Qwen38`` / ``HybridCache`` / ``forward_step`` / ``generate`` on sm_100a kernels.

Public surface and semantics follow reference/qwen38_inference.py ("REF"):
``HybridCache`` (REF:4786-4818), ``_token_batch`` (REF:4821-4841), ``Qwen38.new_cache``
(REF:4966-4983), ``_reserve`` (REF:4985-5001), ``forward_step`` (REF:5004-5099),
``generate`` (REF:5102-5147) and the module functions (REF:5150-5157). Every validation
error is raised before any cache mutation except growth, as in REF.

Everything the GPU computes goes through ``libqw200.so`` (include/qw200.h); torch provides
device memory, the current stream, pinned host staging and CUDA graphs. There is no CPU
path: construction fails unless the device is a CUDA compute capability 10.x GPU and the
library loads.
"""
from __future__ import annotations

import collections
import dataclasses
import itertools
import json
import math
import weakref
from pathlib import Path

import numpy as np
import torch

from . import _lib, ops
from .config import HybridConfig, nested_layers, qwen38_27b, random_weights, rope_table

PAGE = 64


@dataclasses.dataclass
class HybridCache:
    """Per-request keys, values, convolution history, and recurrent state (REF:4786-4818).

    Slots are stable across calls; ``lengths`` count tokens already consumed. KV pools are
    ``[S*capacity + 64, nkv, d]`` bf16 with page 0 reserved; ``conv[i]`` is ``[S, C, 3]``
    bf16 and ``recurrent[i]`` is ``[S, HV, dv, dk]`` fp32. Growth replaces the KV tensors.
    Do not mutate a cache concurrently from multiple calls.
    """
    owner: int
    lengths: list
    capacity: int
    max_context: int
    kv: dict
    conv: dict
    recurrent: dict

    def clone(self):
        return HybridCache(self.owner, self.lengths.copy(), self.capacity, self.max_context,
                           {i: (k.clone(), v.clone()) for i, (k, v) in self.kv.items()},
                           {i: x.clone() for i, x in self.conv.items()},
                           {i: x.clone() for i, x in self.recurrent.items()})

    @torch.inference_mode()
    def reset(self, request_indices=None):
        slots = list(range(len(self.lengths))) if request_indices is None else list(request_indices)
        if len(set(slots)) != len(slots) or any(i < 0 or i >= len(self.lengths) for i in slots):
            raise ValueError("Invalid or duplicate cache slots")
        for slot in slots:
            self.lengths[slot] = 0
            for state in self.conv.values():
                state[slot].zero_()
            for state in self.recurrent.values():
                state[slot].zero_()


def _token_batch(input_ids):
    """REF:4821-4841: normalize input to rows of int and report whether it was flat."""
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
        if set(map(type, row)) != {int}:  # exactly int (no bool, float or numpy scalars)
            raise ValueError("Token IDs must be integers")
        result.append(list(row))
    return result, single


def build_metadata(slots, prefixes, lens, capacity, attn_tile=128):
    """All per-call indices as one int32 array (uploaded with a single H2D copy).

    Bit-exact with REF:5023-5044 for the quantities REF builds: positions = prefix + j,
    locations = 64 + slot*capacity + prefix + j, cu_seqlens, state indices, has_initial.
    Adds the kernels' own indices: kv_base = 64 + slot*capacity (first cache row of the
    request; REF's page table maps page j of slot s to page 1 + s*capacity/64 + j, so the
    rows of a request are contiguous), seq_len = prefix + n, last row per request, and the
    attention tiles (request, first query) ordered longest-first.
    """
    B = len(lens)
    lens_a = np.asarray(lens, dtype=np.int64)
    pre_a = np.asarray(prefixes, dtype=np.int64)
    slot_a = np.asarray(slots, dtype=np.int64)
    cu = np.zeros(B + 1, dtype=np.int64)
    np.cumsum(lens_a, out=cu[1:])
    T = int(cu[-1])
    seq_of_tok = np.repeat(np.arange(B), lens_a)
    j = np.arange(T, dtype=np.int64) - cu[:-1][seq_of_tok]
    positions = pre_a[seq_of_tok] + j
    kv_base = PAGE + slot_a * capacity
    locations = kv_base[seq_of_tok] + positions
    seq_len = pre_a + lens_a
    tiles = [(i, q0, int(pre_a[i]) + q0 + attn_tile) for i in range(B) for q0 in range(0, int(lens_a[i]), attn_tile)]
    tiles.sort(key=lambda x: -x[2])
    tile_arr = np.asarray([(i, q0) for i, q0, _ in tiles], dtype=np.int64).reshape(-1)
    parts = {
        "cu": cu, "slots": slot_a, "has_initial": (pre_a > 0).astype(np.int64), "prefix": pre_a,
        "seq_len": seq_len, "kv_base": kv_base, "last_rows": cu[1:] - 1, "positions": positions,
        "locations": locations, "tiles": tile_arr,
    }
    offs, total = {}, 0
    for k, v in parts.items():
        offs[k] = (total, v.size)
        total += v.size
    packed = np.empty(total, dtype=np.int32)
    for k, v in parts.items():
        o, n = offs[k]
        if n and (v.max() >= 2 ** 31 or v.min() < -(2 ** 31)):
            raise ValueError("cache index exceeds int32")
        packed[o:o + n] = v
    return packed, offs, T


class _BufferArena:
    """Device buffers of dead caches, handed to the next cache of the same shape.

    A new cache (or a grown KV pool) then sits at the addresses of the one it replaces, so
    decode graphs captured on the earlier cache replay on the new one (a graph bakes in
    buffer addresses). Buffers return when their cache is garbage collected or when growth
    replaces a KV pool, and are handed out first in, first out, so each layer of the next
    cache gets the buffer the same layer had before. All use is ordered on one stream: a
    returned buffer is only touched by work queued after its previous owner's last use.
    At most ``max_bytes`` (default a quarter of device memory) are held.
    """

    def __init__(self, device, max_bytes=None):
        self.device = device
        if max_bytes is None:
            max_bytes = (torch.cuda.get_device_properties(device).total_memory // 4
                         if torch.device(device).type == "cuda" else 1 << 30)
        self.max_bytes = max_bytes
        self.held = 0
        self.free = collections.defaultdict(collections.deque)

    def take(self, shape, dtype, zero):
        q = self.free.get((tuple(shape), dtype))
        if q:
            t = q.popleft()
            self.held -= t.numel() * t.element_size()
            if zero:
                t.zero_()
            return t
        return (torch.zeros if zero else torch.empty)(tuple(shape), dtype=dtype, device=self.device)

    def give(self, tensors):
        for t in tensors:
            nbytes = t.numel() * t.element_size()
            if self.held + nbytes <= self.max_bytes:
                self.free[(tuple(t.shape), t.dtype)].append(t)
                self.held += nbytes


class _Staging:
    """Pinned host buffers for metadata uploads, reused once their copy has completed."""

    def __init__(self):
        self.bufs = [None, None]
        self.events = [None, None]
        self.i = 0

    def upload(self, arr: np.ndarray, device, dst: torch.Tensor | None = None) -> torch.Tensor:
        """Copy ``arr`` (int32) to the device without blocking the host: into ``dst`` when
        given (contiguous int32 of arr.size elements), else into a new device tensor."""
        self.i ^= 1
        k = self.i
        if self.events[k] is not None:
            self.events[k].synchronize()
        if self.bufs[k] is None or self.bufs[k].numel() < arr.size:
            self.bufs[k] = torch.empty(max(arr.size, 4096) * 2, dtype=torch.int32, pin_memory=True)
        host = self.bufs[k][:arr.size]
        host.numpy()[:] = arr
        dev = torch.empty(arr.size, dtype=torch.int32, device=device) if dst is None else dst
        dev.copy_(host, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self.events[k] = ev
        return dev


def _check_device(device):
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("CUDA is required")
    if not torch.cuda.is_available():
        raise ValueError("CUDA is required")
    if torch.cuda.get_device_capability(device)[0] != 10:
        raise ValueError("This build supports NVIDIA SM100/SM103 only")
    return device


def load_checkpoint_config(path) -> HybridConfig:
    """``config.json["text_config"]`` of a checkpoint directory (REF:4861), checked as REF
    checks it apart from the fixed 27B sizes (checkpoint.validate_text_config)."""
    from .checkpoint import validate_text_config
    c = json.loads((Path(path) / "config.json").read_text())
    c = c.get("text_config", c)
    validate_text_config(c)
    return HybridConfig.from_text_config(c)


class Qwen38:
    """Hybrid Gated-DeltaNet / gated-GQA decoder on one B200.

    ``Qwen38(model_path, device="cuda:0", max_context=None)`` as in REF:4848. With
    ``model_path=None`` the weights are seeded N(0, 0.02) random init of ``config``
    (default: the 27B geometry), generated on the device; ``weights=`` takes a flat dict
    in the layout of :func:`qwen38_inference_b200.config.weight_shapes`.
    """

    @torch.inference_mode()
    def __init__(self, model_path=None, device="cuda:0", max_context=None, *, config: HybridConfig | None = None,
                 seed: int = 0, weights: dict | None = None, norm_mode: str = "random", tensor_parallel=None):
        self.device = _check_device(device)
        torch.cuda.set_device(self.device)
        _lib.load()  # fail loudly if the native library is missing
        self.path = Path(model_path) if model_path is not None else None
        if self.path is not None:
            cfg = load_checkpoint_config(self.path)
        else:
            cfg = config or qwen38_27b()
        # head-wise tensor parallelism (a torch.distributed process group, or True for the
        # default group): this process holds one rank's heads; see tensor_parallel.py
        self.tp = None
        shard = None
        if tensor_parallel is not None and tensor_parallel is not False:
            from .tensor_parallel import TensorParallel
            self.tp = TensorParallel(None if tensor_parallel is True else tensor_parallel, cfg)
            shard = self.tp.shard
        self.full_cfg = cfg
        self.cfg = self.tp.local_cfg if self.tp is not None else cfg
        self._validate_geometry(self.cfg)
        self.config = cfg.text_config()
        self.dtype = torch.bfloat16
        self.eps = cfg.rms_norm_eps
        self.max_context = cfg.max_position_embeddings if max_context is None else int(max_context)
        if not 1 <= self.max_context <= cfg.max_position_embeddings:
            raise ValueError("max_context must be within the model context limit")
        self.layer_types = cfg.layer_types
        self.eos_token_ids = {cfg.eos_token_id}
        self.page_size = PAGE
        if self.path is not None:
            from .checkpoint import load_weights
            flat = load_weights(self.path, cfg, self.device, shard=shard)
        elif weights is not None:
            flat = {k: (shard(k, v.to(self.device)) if shard else v.to(self.device)) for k, v in weights.items()}
        else:
            flat = random_weights(cfg, seed, device=self.device, norm_mode=norm_mode, shard=shard)
        for k, v in flat.items():
            want = torch.float32 if k.endswith("A_log") else torch.bfloat16
            flat[k] = v.to(device=self.device, dtype=want).contiguous()
        self.layers, g = nested_layers(flat, cfg)
        for kind, w in zip(self.layer_types, self.layers):
            if kind != "full_attention":
                # one projection for [q; k; v; z; b; a]: the small b/a rows ride along with the
                # big GEMM instead of a launch of their own; qkvz and ba stay as row views
                fused = torch.cat([w["qkvz"], w["ba"]], 0)
                w["qkvzba"] = fused
                w["qkvz"], w["ba"] = fused[:self.cfg.qkvz_dim], fused[self.cfg.qkvz_dim:]
        self.embedding, self.final_norm, self.lm_head = g["embedding"], g["final_norm"], g["lm_head"]
        self.rotary_dim = cfg.rotary_dim
        self.rope = rope_table(cfg, self.max_context, self.device)
        self._arena = _BufferArena(self.device)
        from .engine import Engine
        self._engine = Engine(self)

    def enable_peer_allreduce(self):
        """Tensor parallelism only: decode projections all-reduce through the ranks' peer
        buffers inside their GEMM kernel instead of NCCL (collective: every rank calls it)."""
        if self.tp is None:
            raise ValueError("enable_peer_allreduce needs a tensor-parallel model")
        self.tp.enable_peer_buffers(self.cfg.hidden_size, self.device)
        self._engine.graphs.clear()  # graphs captured on the NCCL path

    def check_device_error(self):
        """Wait for the calls queued so far and raise :class:`QwError` naming the failure if a
        kernel recorded one (a bounded wait that gave up, an index outside its range).
        ``forward_step`` also raises at its start for a failure of an earlier call that has
        already reached the host, and ``generate`` checks at each of its token reads."""
        self._engine.check_device_error(block=True)

    def close(self):
        """Release what outlives a call: captured graphs (they may hold NCCL calls) and the
        peer buffers of tensor parallelism. Collective under tensor parallelism."""
        self._engine.graphs.clear()
        if self.tp is not None:
            self.tp.close_peer_buffers()

    @staticmethod
    def _validate_geometry(c: HybridConfig):
        ok = (c.linear_key_head_dim == 128 and c.linear_value_head_dim == 128 and c.linear_conv_kernel_dim == 4
              and c.linear_num_value_heads % c.linear_num_key_heads == 0 and c.head_dim in (64, 128, 256)
              and c.num_attention_heads % c.num_key_value_heads == 0 and c.hidden_size % 8 == 0
              and c.rotary_dim % 2 == 0 and (c.rotary_dim // 2) % (c.head_dim // 32) == 0)
        if not ok:
            raise ValueError("Unsupported hybrid geometry for the sm_100a kernels (GDN heads must be 128-d)")

    # ------------------------------------------------------------------ cache (REF:4966-5001)
    @torch.inference_mode()
    def new_cache(self, batch_size=1, initial_capacity=256, max_context=None):
        c = self.cfg
        if not isinstance(batch_size, int) or batch_size < 1:
            raise ValueError("batch_size must be a positive integer")
        limit = self.max_context if max_context is None else int(max_context)
        if not 1 <= limit <= self.max_context or initial_capacity < 1:
            raise ValueError("Invalid cache capacity/context limit")
        capacity = math.ceil(min(initial_capacity, limit) / PAGE) * PAGE
        kv, conv, recurrent = {}, {}, {}
        take = self._arena.take
        for i, kind in enumerate(self.layer_types):
            if kind == "full_attention":
                shape = (batch_size * capacity + PAGE, c.num_key_value_heads, c.head_dim)
                kv[i] = (take(shape, self.dtype, True), take(shape, self.dtype, True))
            else:
                conv[i] = take((batch_size, c.conv_dim, c.linear_conv_kernel_dim - 1), self.dtype, True)
                recurrent[i] = take((batch_size, c.linear_num_value_heads, c.linear_value_head_dim,
                                     c.linear_key_head_dim), torch.float32, True)
        cache = HybridCache(id(self), [0] * batch_size, capacity, limit, kv, conv, recurrent)
        # the buffers the cache holds when it dies go back to the arena (growth updates the box)
        box = [t for pair in kv.values() for t in pair] + list(conv.values()) + list(recurrent.values())
        cache._arena_box = box
        weakref.finalize(cache, self._arena.give, box)
        return cache

    def _reserve(self, cache, needed):
        if needed > cache.max_context:
            raise ValueError(f"Context limit exceeded: {needed} > {cache.max_context}")
        if needed <= cache.capacity:
            return
        capacity = math.ceil(min(cache.max_context, max(needed, cache.capacity * 2)) / PAGE) * PAGE
        S = len(cache.lengths)
        # pinned staging: the host does not wait for earlier work before queuing the growth
        arr = np.asarray(cache.lengths, dtype=np.int32)
        staging = getattr(self._engine, "staging", None)
        lengths = staging.upload(arr, self.device) if staging is not None else torch.from_numpy(arr).to(self.device)
        new_kv = {}
        box = getattr(cache, "_arena_box", None)
        for i, (k_old, v_old) in cache.kv.items():
            shape = (S * capacity + PAGE,) + tuple(k_old.shape[1:])
            new_kv[i] = (self._arena.take(shape, self.dtype, False), self._arena.take(shape, self.dtype, False))
        if new_kv:  # every layer's pools in one launch
            ops.kv_grow_layers(list(cache.kv.values()), list(new_kv.values()), lengths, S, cache.capacity, capacity)
        old = [t for pair in cache.kv.values() for t in pair]
        cache.kv = new_kv
        cache.capacity = capacity
        if box is not None:
            # the replaced pools leave the cache's box and return to the arena
            ids = {id(t) for t in old}
            box[:] = [t for t in box if id(t) not in ids] + [t for pair in new_kv.values() for t in pair]
            self._arena.give(old)

    # ------------------------------------------------------------------ forward (REF:5004-5099)
    @torch.inference_mode()
    def forward_step(self, input_ids, kv_cache, *, request_indices=None, return_all_logits=False):
        """Consume unpadded token sequences and mutate kv_cache; return fp32 logits
        ``[active_requests, vocab]`` (or ``[total_tokens, vocab]`` with return_all_logits)."""
        rows, _ = _token_batch(input_ids)
        cache = kv_cache
        if not isinstance(cache, HybridCache) or cache.owner != id(self):
            raise ValueError("kv_cache must have been created by this model")
        slots = list(range(len(cache.lengths))) if request_indices is None else list(request_indices)
        if len(slots) != len(rows) or len(set(slots)) != len(slots) or any(
                type(s) is not int or s < 0 or s >= len(cache.lengths) for s in slots):
            raise ValueError("request_indices must identify one distinct cache slot per input sequence")
        lens = [len(r) for r in rows]
        vocab = self.cfg.vocab_size
        try:  # one C-level pass over the ids (a prefill call holds tens of thousands)
            flat = np.fromiter(itertools.chain.from_iterable(rows), dtype=np.int64, count=sum(lens))
        except OverflowError:  # beyond int64, so outside the vocabulary too
            raise ValueError("Token ID outside model vocabulary") from None
        if int(flat.min()) < 0 or int(flat.max()) >= vocab:
            raise ValueError("Token ID outside model vocabulary")
        prefixes = [cache.lengths[s] for s in slots]
        lengths = [p + n for p, n in zip(prefixes, lens)]
        self._reserve(cache, max(lengths))
        is_decode = all(n == 1 and p > 0 for n, p in zip(lens, prefixes))
        logits = self._engine.forward(flat, slots, prefixes, lens, cache, is_decode, return_all_logits)
        for slot, length in zip(slots, lengths):
            cache.lengths[slot] = length
        return logits

    # ------------------------------------------------------------------ generate (REF:5102-5147)
    @torch.inference_mode()
    def generate(self, input_ids, *, max_new_tokens=None, eos_token_ids=None, prefill_chunk_size=512):
        """Greedy generation until each request emits EOS (included), REF:5102-5147."""
        rows, single = _token_batch(input_ids)
        if max_new_tokens is not None and (type(max_new_tokens) is not int or max_new_tokens < 0):
            raise ValueError("max_new_tokens must be a nonnegative integer or None")
        if type(prefill_chunk_size) is not int or prefill_chunk_size < 1:
            raise ValueError("prefill_chunk_size must be a positive integer")
        eos = self.eos_token_ids if eos_token_ids is None else (
            {eos_token_ids} if isinstance(eos_token_ids, int) else set(eos_token_ids))
        if not eos or any(type(t) is not int or t < 0 or t >= self.cfg.vocab_size for t in eos):
            raise ValueError("eos_token_ids must contain valid vocabulary IDs")
        output = [[] for _ in rows]
        if max_new_tokens == 0:
            return output[0] if single else output
        cache = self.new_cache(len(rows))
        if any(len(row) > cache.max_context for row in rows):
            raise ValueError("Input exceeds model context")
        last_logits = {}
        for offset in range(0, max(map(len, rows)), prefill_chunk_size):
            slots = [i for i, row in enumerate(rows) if offset < len(row)]
            chunks = [rows[i][offset:offset + prefill_chunk_size] for i in slots]
            logits = self.forward_step(chunks, cache, request_indices=slots)
            for j, slot in enumerate(slots):
                last_logits[slot] = logits[j]
        active = list(range(len(rows)))
        logits = torch.stack([last_logits[i] for i in active])
        while active:
            # decode steps that can run before the host must look at a token: every active
            # request's remaining context (a step past it would raise) and the most tokens any
            # request still needs
            room = min(cache.max_context - cache.lengths[s] for s in active)
            need = (max(max_new_tokens - len(output[s]) for s in active) if max_new_tokens is not None
                    else math.inf)
            w = min(self.GEN_WINDOW, room, need)
            if w > 1:
                active, logits = self._decode_window(w, need, active, logits, cache, output, eos, max_new_tokens)
                continue
            tokens = logits.argmax(-1).tolist()
            self._engine.check_device_error(block=True)  # the read above synchronized the stream
            next_active, next_inputs = [], []
            for slot, token in zip(active, tokens):
                output[slot].append(token)
                if token in eos or (max_new_tokens is not None and len(output[slot]) >= max_new_tokens):
                    continue
                if cache.lengths[slot] >= cache.max_context:
                    raise RuntimeError(
                        f"Request {slot} exhausted context without EOS; produced {len(output[slot])} tokens")
                next_active.append(slot)
                next_inputs.append([token])
            active = next_active
            if active:
                logits = self.forward_step(next_inputs, cache, request_indices=active)
        return output[0] if single else output

    # decode steps queued back to back inside generate between two host reads of the tokens
    GEN_WINDOW = 8

    def _decode_window(self, w, need, active, logits, cache, output, eos, max_new_tokens):
        """``w`` greedy steps of every request in ``active`` with the tokens kept on the device
        (each step's argmax is the next step's input), then one host read of all ``w`` token
        rows, replayed through REF's per-step bookkeeping (REF:5133-5146): a request stops at
        EOS or at max_new_tokens and its later tokens are dropped. The cache belongs to this
        generate call, so the steps a finished request ran past its end change nothing the
        caller sees; w never exceeds any request's remaining context, so REF's exhaustion
        error can only arise at a window boundary, where the step-by-step loop raises it.
        Returns the requests still generating and their logits."""
        toks = []
        for j in range(w):
            t = logits.argmax(-1)
            toks.append(t)
            if j + 1 < w or w < need:  # the last step feeds no one when every request is done
                logits = self._decode_device_tokens(t, cache, active)
        rows = torch.stack(toks).tolist()  # the window's only device -> host read
        self._engine.check_device_error(block=True)
        pos = {s: k for k, s in enumerate(active)}
        alive = list(active)
        for j in range(w):
            nxt = []
            for s in alive:
                output[s].append(rows[j][pos[s]])
                if rows[j][pos[s]] in eos or (max_new_tokens is not None and len(output[s]) >= max_new_tokens):
                    continue
                nxt.append(s)
            alive = nxt
            if not alive:
                break
        if alive and len(alive) < len(active):
            logits = logits[torch.tensor([pos[s] for s in alive], device=logits.device)]
        return alive, logits

    def _decode_device_tokens(self, tokens, cache, slots):
        """forward_step for one token per slot whose ids are already on the device (an argmax
        over the vocabulary, so always valid): the engine copies them into its input on the
        device instead of uploading host ids."""
        prefixes = [cache.lengths[s] for s in slots]
        lengths = [p + 1 for p in prefixes]
        self._reserve(cache, max(lengths))
        n = len(slots)
        logits = self._engine.forward([0] * n, slots, prefixes, [1] * n, cache, True, False, dev_tokens=tokens)
        for slot, length in zip(slots, lengths):
            cache.lengths[slot] = length
        return logits


def forward_step(model, input_ids, kv_cache, **kwargs):
    """Functional form of Qwen38.forward_step (REF:5150-5152)."""
    return model.forward_step(input_ids, kv_cache, **kwargs)


def generate(model, input_ids, **kwargs):
    """Functional form of Qwen38.generate (REF:5155-5157)."""
    return model.generate(input_ids, **kwargs)


def new_cache(model, batch_size=1, initial_capacity=256, max_context=None):
    """Module-level cache factory looked up by the reference benchmark (benchmark.py:167-171)."""
    return model.new_cache(batch_size, initial_capacity=initial_capacity, max_context=max_context)
