"""The layer loop of ``forward_step`` on the sm_100a kernels (REF:5045-5099).

Prefill (any call that is not pure decode, REF:5027) runs per layer:
  norm -> [attention: qkv GEMM with q/k norm + RoPE + KV store in its epilogue, varlen
           attention (gated), o GEMM]
       or [GDN: one qkvz|ba GEMM, conv + split + L2 norm, chunked delta rule (gating
           fused, state in place), gated RMSNorm, out GEMM]
  -> add-norm -> gate_up GEMM with fused SwiGLU -> down GEMM
then the final add-norm on the selected rows and the lm_head GEMM writing fp32 logits.
Decode replaces the GDN middle by one fused kernel and attention by split-KV decode. Decode
calls and prefill calls of up to 2048 tokens are replayed from a CUDA graph per (launch
shape, cache buffer addresses) once captured.

All per-call indices travel in one int32 upload (``build_metadata``).
"""
from __future__ import annotations

import collections

import numpy as np
import torch

from . import _lib, ops
from .model import _Staging, build_metadata

BF16 = torch.bfloat16


def proj_stride(c) -> int:
    """Row stride (elements) of the buffer that holds a layer's input projection (attention
    qkv or GDN qkvz|ba): the wider of the two, rounded up to 8 elements (16 bytes) for the
    vector and TMA reads of the kernels that take its column blocks (an 8-way tensor-parallel
    rank's qkvz|ba is 2060 wide)."""
    return -(-max(c.qkv_dim, c.qkvz_dim + c.ba_dim) // 8) * 8


class Engine:
    def __init__(self, model):
        self.m = model
        self.c = model.cfg
        self.dev = model.device
        self.ws = ops.Workspace(self.dev, 1 << 20)
        self.staging = _Staging()
        self.graphs = collections.OrderedDict()
        self.use_graphs = True
        self.replays = 0  # calls served by a captured graph
        self._err_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self._err_np = self._err_host.numpy()  # host view: read and cleared outside inference mode too
        self._err_event = None

    # ------------------------------------------------------------------ helpers
    def _decode_splits(self, capacity):
        """Key splits of decode attention: one per 512 slots of capacity, at most 128. A CTA of
        2 warps then streams up to 256 keys per warp, long enough to hide its start-up (27B
        decode steps at B32/1024, B4/8192 and B64/512 tokens of context measured 0.2-0.7 ms
        faster than with 128-slot splits; equal at B1/16384)."""
        return int(min(128, max(1, (capacity + 511) // 512)))

    def _meta_views(self, dev, offs):
        return {k: dev[o:o + n] for k, (o, n) in offs.items()}

    # ------------------------------------------------------------------ device errors
    def check_device_error(self, block=False):
        """Raise :class:`QwError` if a kernel of an earlier call recorded a device-side failure
        (a bounded wait that gave up, an index outside its range). Every call queues a copy of
        the library's error word into pinned memory after its kernels; this reads it once that
        copy has landed (at once when ``block``, else only if it already has), and on a nonzero
        word takes and clears it (``qw_take_device_error``, which also resets the GEMM's ticket
        counters) before raising."""
        ev = self._err_event
        if ev is None or not (block or ev.query()):
            return
        if block:
            ev.synchronize()
        self._err_event = None
        if int(self._err_np[0]) != 0:
            code = _lib.take_device_error()
            self._err_np[0] = 0
            raise _lib.QwError(f"device-side failure in an earlier forward_step: {_lib.device_error_name(code)}")

    def _peek_device_error(self):
        _lib.call("qw_peek_device_error_async", self._err_host.data_ptr(), ops._stream())
        ev = torch.cuda.Event()
        ev.record()
        self._err_event = ev

    # ------------------------------------------------------------------ entry
    def forward(self, flat, slots, prefixes, lens, cache, is_decode, return_all_logits, dev_tokens=None):
        """One forward_step; ``dev_tokens`` (a device integer tensor of the call's T ids) replaces
        the host ids of ``flat`` when the caller's ids are already on the device. Raises first
        if an earlier call's kernels recorded a device error that has reached the host."""
        self.check_device_error()
        out = self._forward(flat, slots, prefixes, lens, cache, is_decode, return_all_logits, dev_tokens)
        self._peek_device_error()
        return out

    def _forward(self, flat, slots, prefixes, lens, cache, is_decode, return_all_logits, dev_tokens=None):
        packed, offs, T = build_metadata(slots, prefixes, lens, cache.capacity)
        tokens = np.asarray(flat, dtype=np.int32)
        arr = np.concatenate([tokens, packed])
        self.last_h2d_bytes = int(arr.nbytes)
        B = len(slots)
        c = self.c
        pf_splits = 1
        if not is_decode:
            max_keys = max(p + n for p, n in zip(prefixes, lens))
            pf_splits = ops.prefill_attn_splits(c.num_attention_heads, offs["tiles"][1] // 2, max_keys)
        # prefill graphs only on one GPU: capturing a chunk's NCCL calls costs more than its
        # launch sequence, and a chunked prompt changes key at every capacity doubling
        small_prefill = T <= self.GRAPH_MAX_PREFILL_T and self.m.tp is None
        if self.use_graphs and not return_all_logits and (is_decode or small_prefill):
            shape = ("decode", B, T) if is_decode else ("prefill", B, T, tuple(lens), pf_splits)
            return self._graph_call(shape, arr, offs, T, B, max(lens), cache, is_decode, pf_splits, dev_tokens)
        dev = self.staging.upload(arr, self.dev)
        if dev_tokens is not None:
            dev[:T].copy_(dev_tokens)
        md = self._meta_views(dev[T:], offs)
        md["tokens"] = dev[:T]
        return self._run(md, T, B, max(lens), cache, is_decode, return_all_logits, pf_splits=pf_splits)

    # ------------------------------------------------------------------ CUDA graphs
    MAX_GRAPHS = 4  # captured graphs kept, least recently used evicted first
    # prefill calls up to this many tokens also run from graphs: their launch sequence costs
    # more host time than the GPU spends (chunked prefill of one long request, 512 tokens a call)
    GRAPH_MAX_PREFILL_T = 2048

    def _graph_call(self, shape, arr, offs, T, B, max_len, cache, is_decode, pf_splits, dev_tokens=None):
        """Run through a CUDA graph keyed by the call's launch shape and the addresses of every
        cache buffer. A graph bakes in its pointers and grid sizes, so any call with that shape
        on a cache whose buffers sit at exactly those addresses with the same capacity and slot
        count replays it correctly (the per-call indices are device data copied in first),
        including a fresh cache that the allocator placed where a freed one was.

        The first call of a key runs eagerly. The second runs eagerly too and then captures
        the same launch sequence (capture records, it does not execute) with a workspace and
        an index buffer of its own. Later calls copy the new indices in and replay. Under
        tensor parallelism every rank executes the collectives of exactly one forward per call
        whichever of the three paths it takes, so ranks whose keys differ stay in step.
        """
        key = shape + (cache.capacity, len(cache.lengths), tuple(k.data_ptr() for k, _ in cache.kv.values()),
                       tuple(x.data_ptr() for x in cache.recurrent.values()),
                       tuple(x.data_ptr() for x in cache.conv.values()))
        ent = self.graphs.get(key)
        if ent is not None and ent["graph"] is not None:
            if ent["offs"] != offs:
                raise RuntimeError("metadata layout changed for a captured shape")
            self.graphs.move_to_end(key)
            # through pinned memory, so the host queues the replay while earlier work (the
            # call's KV growth) still runs instead of waiting for it in a pageable copy
            self.staging.upload(arr, self.dev, dst=ent["input"])
            if dev_tokens is not None:
                ent["input"][:T].copy_(dev_tokens)
            ent["graph"].replay()
            self.replays += 1
            ops.LAUNCHES[0] += ent["launches"]
            return ent["out"].clone()
        dev_in = self.staging.upload(arr, self.dev)  # kept by the graph of this key
        if dev_tokens is not None:
            dev_in[:T].copy_(dev_tokens)
        md = self._meta_views(dev_in[T:], offs)
        md["tokens"] = dev_in[:T]
        out = self._run(md, T, B, max_len, cache, is_decode, False, self.ws, pf_splits=pf_splits)
        if ent is None:
            self.graphs[key] = {"graph": None}
        else:
            gws = ops.Workspace(self.dev, self.ws.buf.numel())  # sized by the eager run
            g = torch.cuda.CUDAGraph()
            n0 = ops.LAUNCHES[0]
            with torch.cuda.graph(g):
                g_out = self._run(md, T, B, max_len, cache, is_decode, False, gws, pf_splits=pf_splits)
            n_launch = ops.LAUNCHES[0] - n0
            ops.LAUNCHES[0] = n0  # captured launches do not execute
            self.graphs[key] = {"graph": g, "input": dev_in, "out": g_out, "offs": offs, "launches": n_launch,
                                "ws": gws}
        self.graphs.move_to_end(key)
        while len(self.graphs) > self.MAX_GRAPHS:
            self.graphs.popitem(last=False)
        return out

    # ------------------------------------------------------------------ the layer loop
    def run_units(self, flat, slots, prefixes, lens, cache, is_decode, units, hidden, resid):
        """Part of one forward_step's layer loop, eagerly, from a given state: ``units`` =
        (first, last) half-layer units, unit 2i being layer i's mixer (attention or GDN, its
        output projection and the post-mixer add-norm) and unit 2i + 1 its MLP (with the next
        layer's input add-norm, except after the last layer). ``hidden`` (the normalized input
        of unit ``first``) and ``resid`` (the residual stream), bf16 [T, H] on the device, are
        updated in place to the state after unit ``last - 1``: the normalized input of the
        next unit, or after the last layer the down projection's output. The cache is used
        and written as by forward_step, but lengths are not committed. The parity tests feed
        single units the oracle's state this way."""
        packed, offs, T = build_metadata(slots, prefixes, lens, cache.capacity)
        dev = self.staging.upload(np.concatenate([np.asarray(flat, dtype=np.int32), packed]), self.dev)
        md = self._meta_views(dev[T:], offs)
        md["tokens"] = dev[:T]
        pf_splits = 1
        if not is_decode:
            pf_splits = ops.prefill_attn_splits(self.c.num_attention_heads, offs["tiles"][1] // 2,
                                                max(p + n for p, n in zip(prefixes, lens)))
        h, r = self._run(md, T, len(slots), max(lens), cache, is_decode, False, pf_splits=pf_splits, units=units,
                         start=(hidden, resid))
        hidden.copy_(h)
        resid.copy_(r)

    def _run(self, md, T, B, max_len, cache, is_decode, return_all_logits, ws=None, pf_splits=1, units=None,
             start=None):
        m, c, dev = self.m, self.c, self.dev
        tp = m.tp
        ws = self.ws if ws is None else ws
        H = c.hidden_size
        eps = m.eps
        resid = torch.empty(T, H, dtype=BF16, device=dev)
        hidden = torch.empty(T, H, dtype=BF16, device=dev)
        if start is None:
            ops.embed_rmsnorm(md["tokens"], m.embedding, m.layers[0]["input_norm"], resid, hidden, eps)
        else:
            hidden.copy_(start[0])
            resid.copy_(start[1])
        nq, nkv, d = c.num_attention_heads, c.num_key_value_heads, c.head_dim
        Hk, HV, dk, dv = c.linear_num_key_heads, c.linear_num_value_heads, c.linear_key_head_dim, c.linear_value_head_dim
        big = proj_stride(c)
        proj = torch.empty(T, big, dtype=BF16, device=dev)
        mix = torch.empty(T, max(c.attn_out_dim, c.gdn_v_dim), dtype=BF16, device=dev)
        act = torch.empty(T, c.intermediate_size, dtype=BF16, device=dev)
        if not is_decode:
            qb = torch.empty(T, c.gdn_qk_dim, dtype=BF16, device=dev)
            kb = torch.empty(T, c.gdn_qk_dim, dtype=BF16, device=dev)
            vb = torch.empty(T, c.gdn_v_dim, dtype=BF16, device=dev)
        splits = self._decode_splits(cache.capacity)
        fused = is_decode and T <= 64  # weight-streaming projections: split-K sum + add-norm in one kernel
        # tensor parallel: row-parallel projections produce fp32 partial sums, all-reduced in place
        # (decode: inside the projection's kernel through the ranks' peer buffers)
        part = torch.empty(T, H, dtype=torch.float32, device=dev) if tp is not None else None
        peer = tp is not None and tp.peer_bases is not None and fused and all(
            ops.gemm_add_rmsnorm_kernels(T, H, K) == 1 for K in {c.attn_out_dim, c.gdn_v_dim, c.intermediate_size})
        use = [0]  # row-parallel projections so far in this call: the peer slot alternates

        def peer_slot(last=False):
            slot = 2 if last else use[0] % 2
            use[0] += 1
            return slot

        def proj_add_norm(x, wt, norm_w):
            """hidden = x . wt^T, then resid += hidden, hidden = norm(resid)."""
            if peer:
                ops.gemm_add_rmsnorm_tp(x, wt, resid, norm_w, hidden, eps, ws, tp.peer_bases, tp.world, tp.rank,
                                        peer_slot())
            elif tp is not None:
                ops.gemm(x, wt, part, out_kind=ops.OUT_F32, ws=ws)
                tp.all_reduce_(part)
                ops.add_rmsnorm_f32(part, resid, norm_w, hidden, eps)
            elif fused or ops.gemm_add_rmsnorm_workspace_bytes(T, wt.shape[0], wt.shape[1]):
                # weight streaming (decode) or too few tiles (a chunk): split-K partials summed
                # by the add-norm kernel
                ops.gemm_add_rmsnorm(x, wt, resid, norm_w, hidden, eps, ws)
            else:
                ops.gemm(x, wt, hidden, ws=ws)
                ops.add_rmsnorm(hidden, resid, norm_w, eps)

        n_layers = len(m.layers)

        def mixer(i):
            kind, w = m.layer_types[i], m.layers[i]
            if kind == "full_attention":
                qkv = proj[:, :c.qkv_dim]
                kc, vc = cache.kv[i]
                # projection, q/k norm, RoPE and the KV store in one GEMM epilogue (a split-K
                # product and one finishing kernel for decode and sparse-tile chunks)
                ops.gemm_qkv_rope_store(hidden, w["qkv"], qkv, nq, nkv, d, w["q_norm"], w["k_norm"], m.rope,
                                        md["positions"], md["locations"], kc, vc, eps, ws)
                att = mix[:, :c.attn_out_dim]
                if is_decode:
                    ops.attn_decode(qkv, B, nq, nkv, d, kc, vc, md["seq_len"], md["kv_base"], cache.capacity, splits,
                                    att, d ** -0.5, ws)
                else:
                    ops.attn_prefill(qkv, nq, nkv, d, kc, vc, md["tiles"], md["cu"], md["prefix"], md["kv_base"],
                                     att, d ** -0.5, splits=pf_splits, ws=ws)
                proj_add_norm(att, w["out"], w["post_norm"])
            else:
                ops.gemm(hidden, w["qkvzba"], proj[:, :c.qkvz_dim + c.ba_dim], ws=ws)
                qkvz, ba = proj[:, :c.qkvz_dim], proj[:, c.qkvz_dim:c.qkvz_dim + c.ba_dim]
                y = mix[:, :c.gdn_v_dim]
                if is_decode:
                    ops.gdn_decode(qkvz, ba, w["conv"], cache.conv[i], cache.recurrent[i], md["slots"], B, w["A_log"],
                                   w["dt_bias"], w["norm"], y, Hk, HV, dk, dv, eps)
                else:
                    ops.conv_prefill(qkvz, w["conv"], cache.conv[i], md["cu"], md["slots"], md["has_initial"], B,
                                     max_len, qb, kb, vb, c.gdn_qk_dim, c.gdn_v_dim, dk)
                    ops.gdn_prefill(qb, kb, vb, ba, w["A_log"], w["dt_bias"], md["cu"], md["slots"], B,
                                    cache.recurrent[i], qkvz[:, c.conv_dim:], w["norm"], y, Hk, HV, dk, dv,
                                    dk ** -0.5, eps)
                proj_add_norm(y, w["out"], w["post_norm"])

        def mlp(i):
            w = m.layers[i]
            ops.gemm(hidden, w["gate_up"], act, out_kind=ops.OUT_SWIGLU, ws=ws)
            if i + 1 < n_layers:
                proj_add_norm(act, w["down"], m.layers[i + 1]["input_norm"])  # the next layer's input norm
            elif peer:
                ops.gemm_add_rmsnorm_tp(act, w["down"], None, None, hidden, eps, ws, tp.peer_bases, tp.world, tp.rank,
                                        peer_slot(last=True), round_only=True)
            elif tp is not None:
                ops.gemm(act, w["down"], part, out_kind=ops.OUT_F32, ws=ws)
                tp.all_reduce_(part)
                ops.round_f32_bf16(part, hidden)
            else:
                ops.gemm(act, w["down"], hidden, ws=ws)

        lo, hi = (0, 2 * n_layers) if units is None else units
        for u in range(lo, hi):
            (mlp if u % 2 else mixer)(u // 2)
        if units is not None:
            return hidden, resid
        rows = None if return_all_logits else md["last_rows"]
        R = T if return_all_logits else B
        fin = torch.empty(R, H, dtype=BF16, device=dev)
        ops.add_rmsnorm_rows(hidden, resid, m.final_norm, fin, eps, rows)
        logits = torch.empty(R, c.vocab_size, dtype=torch.float32, device=dev)
        if tp is None:
            ops.gemm(fin, m.lm_head, logits, out_kind=ops.OUT_F32_OF_BF16, ws=ws)
            return logits
        # vocab-parallel lm_head: each rank's rows, all-gathered rank-major, then reordered
        Vs = m.lm_head.shape[0]
        local = torch.empty(R, Vs, dtype=torch.float32, device=dev)
        ops.gemm(fin, m.lm_head, local, out_kind=ops.OUT_F32_OF_BF16, ws=ws)
        gathered = torch.empty(tp.world * R, Vs, dtype=torch.float32, device=dev)
        tp.all_gather_rows(local, gathered)
        ops.gather_vocab_shards(gathered.view(tp.world, R, Vs), logits)
        return logits
