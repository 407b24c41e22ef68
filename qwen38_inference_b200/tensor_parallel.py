"""Head-wise tensor parallelism of the hybrid model over the GPUs of one node.

The long-context case (one request, e.g. 131071 tokens prefilled in 512-token chunks, then
decode) does not shard by request, so its heads are split across ranks, one process per
GPU, with NCCL over NVLink for the exchanges:

* column-parallel (each rank owns whole heads or rows and computes them locally):
  - attention ``qkv``: query heads ``[r*nq/G, (r+1)*nq/G)`` with their interleaved gates,
    and their KV heads. When G exceeds the KV head count each KV head is replicated on the
    G/nkv ranks whose query heads use it.
  - GDN ``qkvz``: QK heads ``[r*Hk/G, ...)`` and value heads ``[r*HV/G, ...)``. They stay
    contiguous because value head hv uses QK head hv // (HV/Hk).
  - ``ba``, ``conv``, ``A_log``, ``dt_bias``: the slices of the rank's value and QK heads.
  - MLP ``gate_up``: rows ``[r*I/G, ...)`` of the gate half and of the up half.
  - ``lm_head``: vocabulary rows ``[r*V/G, ...)``.
* row-parallel (each rank holds a column slice, and the outputs are summed):
  attention ``o_proj``, GDN ``out_proj`` and MLP ``down``. Each rank computes an fp32 partial
  product and the ``[T, hidden]`` fp32 sum is rounded to bf16 once, so the result equals the
  one-GPU projection up to fp32 summation order. Prefill sums with an NCCL all-reduce;
  decode (up to 64 rows), once ``enable_peer_buffers`` has run, sums inside the projection's
  own kernel: its last CTAs read the other ranks' rows from their buffers over NVLink
  (CUDA IPC) and apply the residual add-norm.
* replicated: the embedding, every RMSNorm weight, the residual stream and the hidden state.

The conv state, recurrent state and KV cache of each rank hold only its own heads. The
logits of the vocabulary shards are all-gathered and put back in vocabulary order.

Every rank must make the same ``forward_step`` calls with the same arguments, in the same
order, because each call runs the same sequence of collectives. The reference runs on one
GPU and has no counterpart to this module.
"""
from __future__ import annotations

import dataclasses

import torch

from .config import HybridConfig


@dataclasses.dataclass(frozen=True)
class ShardSpec:
    """The rank's slice of every sharded dimension of the geometry ``cfg``."""
    rank: int
    world: int
    cfg: HybridConfig

    # --------------------------------------------------------------- attention heads
    @property
    def nq(self) -> int:
        return self.cfg.num_attention_heads // self.world

    @property
    def nkv(self) -> int:
        c = self.cfg
        return c.num_key_value_heads // self.world if c.num_key_value_heads >= self.world else 1

    @property
    def kv_head0(self) -> int:
        """First (global) KV head held by this rank."""
        c = self.cfg
        if c.num_key_value_heads >= self.world:
            return self.rank * self.nkv
        group = c.num_attention_heads // c.num_key_value_heads
        return (self.rank * self.nq) // group

    # --------------------------------------------------------------- GDN heads, MLP, vocab
    @property
    def hk(self) -> int:
        return self.cfg.linear_num_key_heads // self.world

    @property
    def hv(self) -> int:
        return self.cfg.linear_num_value_heads // self.world

    @property
    def inter(self) -> int:
        return self.cfg.intermediate_size // self.world

    @property
    def vocab(self) -> int:
        return self.cfg.vocab_size // self.world


def check_shardable(cfg: HybridConfig, world: int) -> None:
    """Raise ValueError unless ``cfg`` splits evenly over ``world`` ranks."""
    c = cfg
    if world < 1:
        raise ValueError("tensor-parallel world size must be >= 1")
    bad = []
    for name, n in (("num_attention_heads", c.num_attention_heads), ("linear_num_key_heads", c.linear_num_key_heads),
                    ("linear_num_value_heads", c.linear_num_value_heads), ("intermediate_size", c.intermediate_size),
                    ("vocab_size", c.vocab_size)):
        if n % world:
            bad.append(name)
    nkv, nq = c.num_key_value_heads, c.num_attention_heads
    if nkv >= world:
        if nkv % world:
            bad.append("num_key_value_heads")
    else:
        group, nq_l = nq // nkv, nq // world
        if world % nkv or group % max(nq_l, 1):  # a rank's query heads must share one KV head
            bad.append("num_key_value_heads")
    if c.vocab_size % world == 0 and (c.vocab_size // world) % 4:
        bad.append("vocab_size (shard not a multiple of 4)")
    if bad:
        raise ValueError(f"geometry does not split over {world} ranks: {', '.join(bad)}")


def shard_config(cfg: HybridConfig, world: int) -> HybridConfig:
    """The per-rank geometry: head counts and MLP width divided by ``world`` (KV heads
    replicated when fewer than ``world``). ``vocab_size`` stays the full vocabulary (the
    embedding and the token checks use it); the rank's lm_head holds ``vocab_size/world``
    rows."""
    check_shardable(cfg, world)
    sp = ShardSpec(0, world, cfg)
    return dataclasses.replace(cfg, num_attention_heads=sp.nq, num_key_value_heads=sp.nkv,
                               linear_num_key_heads=sp.hk, linear_num_value_heads=sp.hv,
                               intermediate_size=sp.inter)


def _rows(t, *ranges):
    return torch.cat([t[a:b] for a, b in ranges], 0) if len(ranges) > 1 else t[ranges[0][0]:ranges[0][1]]


def shard_tensor(name: str, t: torch.Tensor, sp: ShardSpec) -> torch.Tensor:
    """The rank's slice of the full weight ``name`` (layout of ``config.weight_shapes``),
    as a new contiguous tensor."""
    c, r = sp.cfg, sp.rank
    key = name.rsplit(".", 1)[-1]
    layer_kind = None
    if name.startswith("layers."):
        layer_kind = c.layer_types[int(name.split(".")[1])]
    if name == "lm_head":
        out = t[r * sp.vocab:(r + 1) * sp.vocab]
    elif key == "gate_up":
        I, i0 = c.intermediate_size, r * sp.inter
        out = _rows(t, (i0, i0 + sp.inter), (I + i0, I + i0 + sp.inter))
    elif key == "down":
        out = t[:, r * sp.inter:(r + 1) * sp.inter]
    elif layer_kind == "full_attention" and key == "qkv":
        d, nq, nkv = c.head_dim, c.num_attention_heads, c.num_key_value_heads
        q0 = r * sp.nq * 2 * d  # [q | gate] interleaved per query head
        k0 = nq * 2 * d + sp.kv_head0 * d
        v0 = nq * 2 * d + nkv * d + sp.kv_head0 * d
        out = _rows(t, (q0, q0 + sp.nq * 2 * d), (k0, k0 + sp.nkv * d), (v0, v0 + sp.nkv * d))
    elif layer_kind == "full_attention" and key == "out":
        d = c.head_dim
        out = t[:, r * sp.nq * d:(r + 1) * sp.nq * d]
    elif key in ("qkvz", "conv"):
        dk, dv, Hk, HV = c.linear_key_head_dim, c.linear_value_head_dim, c.linear_num_key_heads, c.linear_num_value_heads
        qk = Hk * dk
        q0, k0, v0 = r * sp.hk * dk, qk + r * sp.hk * dk, 2 * qk + r * sp.hv * dv
        ranges = [(q0, q0 + sp.hk * dk), (k0, k0 + sp.hk * dk), (v0, v0 + sp.hv * dv)]
        if key == "qkvz":
            z0 = 2 * qk + HV * dv + r * sp.hv * dv
            ranges.append((z0, z0 + sp.hv * dv))
        out = _rows(t, *ranges)
    elif key == "ba":
        HV, h0 = c.linear_num_value_heads, r * sp.hv
        out = _rows(t, (h0, h0 + sp.hv), (HV + h0, HV + h0 + sp.hv))
    elif key in ("A_log", "dt_bias"):
        out = t[r * sp.hv:(r + 1) * sp.hv]
    elif layer_kind == "linear_attention" and key == "out":
        dv = c.linear_value_head_dim
        out = t[:, r * sp.hv * dv:(r + 1) * sp.hv * dv]
    else:  # embedding, final_norm, input_norm, post_norm, q_norm, k_norm, norm
        out = t
    # a slice is copied out, so the shard does not keep the full tensor's storage alive
    return t if out is t else out.clone(memory_format=torch.contiguous_format)


class TensorParallel:
    """The process group and this rank's shard of one model (``Qwen38(tensor_parallel=...)``)."""

    def __init__(self, group, cfg: HybridConfig):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.spec = ShardSpec(self.rank, self.world, cfg)
        self.local_cfg = shard_config(cfg, self.world)
        self.full_cfg = cfg

    def shard(self, name, t):
        return shard_tensor(name, t, self.spec)

    # ------------------------------------------------------------------ peer buffers
    peer_bases = None  # int64 device tensor of every rank's peer buffer (decode all-reduce)

    def enable_peer_buffers(self, hidden_size: int, device) -> None:
        """Allocate this rank's peer buffer (CUDA IPC), exchange handles with the group and
        map the other ranks' buffers, so that decode projections all-reduce inside their
        GEMM kernel (``ops.gemm_add_rmsnorm_tp``) instead of through NCCL. Collective: every
        rank calls it."""
        import ctypes as C
        from . import _lib
        L = _lib.load()
        nbytes = int(L.qw_tp_buffer_bytes(hidden_size))
        own = C.c_void_p()
        handle = C.create_string_buffer(64)
        _lib.check(L.qw_ipc_alloc(nbytes, C.byref(own), handle), "qw_ipc_alloc")
        handles = [None] * self.world
        self.dist.all_gather_object(handles, handle.raw, group=self.group)
        bases, opened = [], []
        for r, h in enumerate(handles):
            if r == self.rank:
                bases.append(own.value)
                continue
            p = C.c_void_p()
            _lib.check(L.qw_ipc_open(C.create_string_buffer(h, 64), C.byref(p)), "qw_ipc_open")
            bases.append(p.value)
            opened.append(p.value)
        self._own_buffer, self._opened = own.value, opened
        self.peer_bases = torch.tensor(bases, dtype=torch.int64, device=device)
        self.dist.barrier(group=self.group)  # every rank maps every buffer before first use

    def close_peer_buffers(self) -> None:
        """Unmap the other ranks' buffers and free this rank's. Collective; call it when no
        kernel of any rank can still use them (after a synchronize), before the group ends."""
        if self.peer_bases is None:
            return
        from . import _lib
        L = _lib.load()
        torch.cuda.synchronize()
        self.dist.barrier(group=self.group)
        for p in self._opened:
            _lib.check(L.qw_ipc_close(p), "qw_ipc_close")
        self.dist.barrier(group=self.group)  # nobody maps this rank's buffer any more
        _lib.check(L.qw_ipc_free(self._own_buffer), "qw_ipc_free")
        self.peer_bases = None

    def _timed(self, name, fn):
        from . import _lib
        prof = _lib.PROFILE
        if prof is None:
            fn()
            return
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        prof.append((name, e0, e1))

    def all_reduce_(self, t: torch.Tensor) -> None:
        """In-place sum over the ranks (NCCL, ordered with the current stream)."""
        if self.world > 1:
            self._timed("qw_nccl_all_reduce", lambda: self.dist.all_reduce(t, group=self.group))

    def all_gather_rows(self, local: torch.Tensor, out: torch.Tensor) -> None:
        """out [G * R, ...] = the ranks' ``local`` [R, ...] tensors, rank-major."""
        if self.world > 1:
            self._timed("qw_nccl_all_gather",
                        lambda: self.dist.all_gather_into_tensor(out, local, group=self.group))
        else:
            out.copy_(local)
