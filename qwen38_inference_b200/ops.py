"""Torch-facing wrappers over the C ABI (include/qw200.h).

Each wrapper checks dtypes, devices and contiguity, passes raw pointers, sizes and the
current CUDA stream to ``libqw200.so``, and raises on any nonzero status. There is no
fallback path: every op runs the sm_100a kernel or fails.
"""
from __future__ import annotations

import torch

from . import _lib

BF16 = torch.bfloat16
OUT_BF16, OUT_F32_OF_BF16, OUT_SWIGLU, OUT_F32 = 0, 1, 2, 3

# Kernels launched through this module (a benchmark's claim of native launches), and an
# optional list that, when set, receives (flops, start_event, end_event, (M, N, K, out_kind))
# per GEMM launch.
LAUNCHES = [0]
PROFILE = None


def _ptr(t):
    return t.data_ptr() if t is not None else None


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _req(t, dtype, name):
    if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dtype != dtype:
        raise TypeError(f"{name} must be a CUDA {dtype} tensor")


class Workspace:
    """A growable device scratch buffer owned by the caller (the library never allocates)."""

    def __init__(self, device, nbytes: int = 0):
        self.device = torch.device(device)
        self.buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=self.device)

    def get(self, nbytes: int) -> torch.Tensor:
        if nbytes > self.buf.numel():
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("workspace must be sized before CUDA-graph capture")
            self.buf = torch.empty(int(nbytes * 1.25) + 256, dtype=torch.uint8, device=self.device)
        return self.buf


def gemm_workspace_bytes(M, N, K, out_kind=OUT_BF16) -> int:
    return int(_lib.load().qw_gemm_workspace_bytes(M, N, K, out_kind))


def gemm(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, *, out_kind: int = OUT_BF16,
         ws: Workspace | None = None) -> torch.Tensor:
    """y = x . w^T (bf16, fp32 accumulation). x [M, K] (row stride >= K), w [N, K]."""
    _req(x, BF16, "x")
    _req(w, BF16, "w")
    if x.dim() != 2 or w.dim() != 2 or x.shape[1] != w.shape[1] or x.stride(1) != 1 or w.stride(1) != 1:
        raise ValueError("gemm expects x [M, K] and w [N, K] with unit inner stride")
    M, K = x.shape
    N = w.shape[0]
    n_out = N // 2 if out_kind == OUT_SWIGLU else N
    odt = torch.float32 if out_kind in (OUT_F32_OF_BF16, OUT_F32) else BF16
    if out is None:
        out = torch.empty(M, n_out, dtype=odt, device=x.device)
    if out.dtype != odt or out.shape != (M, n_out) or out.stride(1) != 1:
        raise ValueError("bad gemm output tensor")
    need = gemm_workspace_bytes(M, N, K, out_kind)
    wsp = None
    if need:
        if ws is None:
            raise ValueError("this gemm shape needs a workspace")
        wsp = ws.get(need)
    prof = PROFILE
    if prof is not None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
    _lib.call("qw_gemm_bf16", x.data_ptr(), w.data_ptr(), out.data_ptr(), M, N, K, x.stride(0), w.stride(0),
              out.stride(0), out_kind, _ptr(wsp), need, _stream())
    if prof is not None:
        e1.record()
        prof.append((2.0 * M * N * K, e0, e1, (M, N, K, out_kind)))
    LAUNCHES[0] += 2 if need else 1
    return out


# ----------------------------------------------------------------------------- norms
def gemm_add_rmsnorm_kernels(M, N, K) -> int:
    """1 when the add-norm of this shape runs inside the GEMM kernel (the condition of the
    tensor-parallel fused path too), else 2."""
    return int(_lib.load().qw_gemm_add_rmsnorm_kernels(M, N, K))


def gemm_add_rmsnorm_workspace_bytes(M, N, K) -> int:
    return int(_lib.load().qw_gemm_add_rmsnorm_workspace_bytes(M, N, K))


def gemm_add_rmsnorm(x, w, resid, norm_w, hidden, eps, ws: Workspace):
    """Projection fused with the add-norm after it: resid += bf16(x . w^T), hidden =
    GemmaRMSNorm(resid) (split-K partials, when the shape takes them, are summed by the
    norm kernel)."""
    _req(x, BF16, "x")
    _req(w, BF16, "w")
    M, K = x.shape
    N = w.shape[0]
    if not (resid.is_contiguous() and hidden.is_contiguous() and resid.shape == (M, N) and hidden.shape == (M, N)):
        raise ValueError("gemm_add_rmsnorm expects contiguous resid and hidden [M, N]")
    need = int(_lib.load().qw_gemm_add_rmsnorm_workspace_bytes(M, N, K))
    buf = ws.get(need)
    LAUNCHES[0] += gemm_add_rmsnorm_kernels(M, N, K)
    _lib.call("qw_gemm_add_rmsnorm", x.data_ptr(), w.data_ptr(), M, N, K, x.stride(0), w.stride(0), resid.data_ptr(),
              norm_w.data_ptr(), hidden.data_ptr(), eps, buf.data_ptr(), need, _stream())


def gemm_add_rmsnorm_tp(x, w, resid, norm_w, hidden, eps, ws: Workspace, peer_bases, world, rank, slot,
                        round_only=False):
    """A tensor-parallel rank's decode row-parallel projection, the all-reduce over the ranks
    through their peer buffers and the residual add-norm (or, ``round_only``, hidden =
    bf16(sum)) in one kernel. ``peer_bases``: int64 device tensor of the ranks' buffer bases."""
    _req(x, BF16, "x")
    _req(w, BF16, "w")
    M, K = x.shape
    N = w.shape[0]
    if not (hidden.is_contiguous() and hidden.shape == (M, N)):
        raise ValueError("gemm_add_rmsnorm_tp expects contiguous hidden [M, N]")
    need = int(_lib.load().qw_gemm_add_rmsnorm_workspace_bytes(M, N, K))
    buf = ws.get(need)
    LAUNCHES[0] += 1
    _lib.call("qw_gemm_add_rmsnorm_tp", x.data_ptr(), w.data_ptr(), M, N, K, x.stride(0), w.stride(0),
              _ptr(resid), _ptr(norm_w), hidden.data_ptr(), eps, buf.data_ptr(), need, peer_bases.data_ptr(), world,
              rank, slot, 1 if round_only else 0, _stream())


def add_rmsnorm_f32(x, resid, norm_w, hidden, eps):
    """resid += bf16(x), hidden = GemmaRMSNorm(resid) with x fp32 [T, H] (an all-reduced
    row-parallel projection), resid and hidden bf16 [T, H] contiguous."""
    T, H = resid.shape
    if not (x.dtype == torch.float32 and x.is_contiguous() and x.shape == (T, H) and resid.is_contiguous()
            and hidden.is_contiguous() and hidden.shape == (T, H)):
        raise ValueError("add_rmsnorm_f32 expects x fp32 [T, H] and contiguous resid/hidden [T, H]")
    LAUNCHES[0] += 1
    _lib.call("qw_add_rmsnorm_f32", x.data_ptr(), 1, 0, T, H, resid.data_ptr(), norm_w.data_ptr(), hidden.data_ptr(),
              eps, _stream())


def round_f32_bf16(x, y):
    """y (bf16) = bf16(x (fp32)), both contiguous with the same number of elements."""
    if not (x.dtype == torch.float32 and y.dtype == BF16 and x.is_contiguous() and y.is_contiguous()
            and x.numel() == y.numel()):
        raise ValueError("round_f32_bf16 expects contiguous fp32 x and bf16 y of one size")
    LAUNCHES[0] += 1
    _lib.call("qw_round_f32_bf16", x.data_ptr(), y.data_ptr(), x.numel(), _stream())


def gather_vocab_shards(src, dst):
    """dst [R, G*Vs] = src [G, R, Vs] reordered so that shard g fills columns g*Vs.."""
    G, R, Vs = src.shape
    if not (src.is_contiguous() and dst.is_contiguous() and dst.shape == (R, G * Vs)
            and src.dtype == torch.float32 and dst.dtype == torch.float32):
        raise ValueError("gather_vocab_shards expects fp32 src [G, R, Vs] and dst [R, G*Vs]")
    LAUNCHES[0] += 1
    _lib.call("qw_gather_vocab_shards", src.data_ptr(), G, R, Vs, dst.data_ptr(), _stream())


def embed_rmsnorm(tokens, table, w, resid_out, hidden_out, eps):
    T = tokens.numel()
    LAUNCHES[0] += 1
    _lib.call("qw_embed_rmsnorm", tokens.data_ptr(), T, table.data_ptr(), table.shape[0], table.shape[1],
              w.data_ptr(), resid_out.data_ptr(), hidden_out.data_ptr(), eps, _stream())


def add_rmsnorm(x, resid, w, eps):
    T, H = x.shape
    LAUNCHES[0] += 1
    _lib.call("qw_add_rmsnorm", x.data_ptr(), resid.data_ptr(), w.data_ptr(), T, H, eps, _stream())


def add_rmsnorm_rows(x, resid, w, out, eps, rows=None):
    T, H = x.shape
    n = rows.numel() if rows is not None else T
    LAUNCHES[0] += 1
    _lib.call("qw_add_rmsnorm_rows", x.data_ptr(), resid.data_ptr(), _ptr(rows), n, T, H, w.data_ptr(),
              out.data_ptr(), eps, _stream())


def gated_rmsnorm(x, z, w, y, HV, D, eps):
    T = x.shape[0]
    LAUNCHES[0] += 1
    _lib.call("qw_gated_rmsnorm", x.data_ptr(), x.stride(0), z.data_ptr(), z.stride(0), w.data_ptr(), y.data_ptr(),
              y.stride(0), T, HV, D, eps, _stream())


# ----------------------------------------------------------------------------- attention
def qk_norm_rope_store(qkv, nq, nkv, d, q_w, k_w, rope, positions, locations, kc, vc, eps):
    T = qkv.shape[0]
    LAUNCHES[0] += 1
    _lib.call("qw_qk_norm_rope_store", qkv.data_ptr(), qkv.stride(0), T, nq, nkv, d, q_w.data_ptr(), k_w.data_ptr(),
              rope.data_ptr(), rope.shape[1], rope.shape[0], positions.data_ptr(), locations.data_ptr(),
              kc.data_ptr(), vc.data_ptr(), kc.shape[0], eps, _stream())


def gemm_qkv_rope_store(x, w, qkv, nq, nkv, d, q_w, k_w, rope, positions, locations, kc, vc, eps, ws: Workspace):
    """The attention input projection fused with q/k norm, RoPE and the KV store:
    qkv[:, q and gate columns] and the cache rows of k and v, as gemm() into qkv followed by
    qk_norm_rope_store() (the k and v columns of qkv are not written)."""
    _req(x, BF16, "x")
    _req(w, BF16, "w")
    M, K = x.shape
    N = w.shape[0]
    if not (qkv.shape[0] == M and qkv.shape[1] >= N and qkv.stride(1) == 1 and x.stride(1) == 1 and w.stride(1) == 1
            and kc.is_contiguous() and vc.is_contiguous() and kc.shape == vc.shape):
        raise ValueError("gemm_qkv_rope_store expects x [M, K], w [N, K], qkv [M, >= N], contiguous K/V caches")
    rd = rope.shape[1]
    need = int(_lib.load().qw_gemm_qkv_workspace_bytes(M, N, K, d, rd))
    buf = ws.get(need) if need else None
    prof = PROFILE
    if prof is not None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
    _lib.call("qw_gemm_qkv_rope_store", x.data_ptr(), w.data_ptr(), qkv.data_ptr(), M, N, K, x.stride(0), w.stride(0),
              qkv.stride(0), nq, nkv, d, q_w.data_ptr(), k_w.data_ptr(), rope.data_ptr(), rd, rope.shape[0],
              positions.data_ptr(), locations.data_ptr(), kc.data_ptr(), vc.data_ptr(), kc.shape[0], eps, _ptr(buf),
              need, _stream())
    if prof is not None:
        e1.record()
        prof.append((2.0 * M * N * K, e0, e1, (M, N, K, "qkv")))
    LAUNCHES[0] += 2 if need else 1
    return qkv


def attn_prefill(qkv, nq, nkv, d, kc, vc, tiles, cu, prefix, kv_base, out, scale, splits=1, ws=None):
    """Causal varlen attention over the cache; qkv [T, ldq] rows, kc/vc [cache_rows, nkv, d].
    ``splits > 1`` divides every tile's keys over that many CTAs (long prefixes) and merges
    the partials, which needs a workspace."""
    if not (kc.is_contiguous() and vc.is_contiguous() and kc.shape == vc.shape and qkv.stride(1) == 1):
        raise ValueError("attn_prefill expects contiguous K/V caches of one shape and unit-stride qkv rows")
    T = qkv.shape[0]
    if splits == 1:
        LAUNCHES[0] += 1
        _lib.call("qw_attn_prefill", qkv.data_ptr(), qkv.stride(0), nq, nkv, d, kc.data_ptr(), vc.data_ptr(),
                  tiles.data_ptr(), tiles.numel() // 2, cu.data_ptr(), prefix.data_ptr(), kv_base.data_ptr(),
                  out.data_ptr(), out.stride(0), scale, T, kc.shape[0], _stream())
        return
    need = int(_lib.load().qw_attn_prefill_split_workspace_bytes(T, nq, d, splits))
    buf = ws.get(need)
    LAUNCHES[0] += 2
    _lib.call("qw_attn_prefill_split", qkv.data_ptr(), qkv.stride(0), nq, nkv, d, kc.data_ptr(), vc.data_ptr(),
              tiles.data_ptr(), tiles.numel() // 2, cu.data_ptr(), prefix.data_ptr(), kv_base.data_ptr(),
              out.data_ptr(), out.stride(0), scale, T, kc.shape[0], splits, buf.data_ptr(), need, _stream())


def prefill_attn_splits(nq, n_tiles, max_keys, sms=148):
    """Key splits for prefill attention: 1 unless heads x tiles leave SMs idle on a long key
    range. Cost model (one 230 KB CTA per SM): waves x (key blocks per split + 4 blocks of
    prologue/merge), minimized over splits with at least 8 key blocks each."""
    units = nq * n_tiles
    blocks = (max_keys + 63) // 64
    if units >= sms or blocks < 32:
        return 1
    best, best_cost = 1, None
    for s in range(1, max(1, blocks // 8) + 1):
        per = -(-blocks // s)
        cost = -(-units * s // sms) * (per + 4)
        if best_cost is None or cost < best_cost:
            best, best_cost = s, cost
    return best


def attn_decode_workspace_bytes(B, nq, d, splits):
    return int(_lib.load().qw_attn_decode_workspace_bytes(B, nq, d, splits))


def attn_decode(qkv, B, nq, nkv, d, kc, vc, seq_len, kv_base, max_len, splits, out, scale, ws: Workspace):
    need = attn_decode_workspace_bytes(B, nq, d, splits)
    buf = ws.get(need)
    LAUNCHES[0] += 2
    _lib.call("qw_attn_decode", qkv.data_ptr(), qkv.stride(0), B, nq, nkv, d, kc.data_ptr(), vc.data_ptr(),
              seq_len.data_ptr(), kv_base.data_ptr(), max_len, splits, out.data_ptr(), out.stride(0), scale,
              buf.data_ptr(), need, _stream())


# ----------------------------------------------------------------------------- gated deltanet
def conv_prefill(x, conv_w, conv_state, cu, slots, has_initial, B, max_len, q_out, k_out, v_out, qk_dim, v_dim,
                 head_dim):
    LAUNCHES[0] += 1
    _lib.call("qw_conv_prefill", x.data_ptr(), x.stride(0), conv_w.data_ptr(), conv_state.data_ptr(), cu.data_ptr(),
              slots.data_ptr(), has_initial.data_ptr(), B, conv_state.shape[0], max_len, q_out.data_ptr(),
              k_out.data_ptr(), v_out.data_ptr(), qk_dim, v_dim, head_dim, _stream())


def gdn_prefill(q, k, v, ba, A_log, dt_bias, cu, slots, B, state, z, norm_w, y, H, HV, dk, dv, scale, eps):
    """Chunked delta rule + gated RMSNorm: y = norm(o) * w * silu(z), o never leaves the SM."""
    T = q.shape[0]
    if not (q.is_contiguous() and k.is_contiguous() and v.is_contiguous() and k.shape[0] == T and v.shape[0] == T
            and q.numel() == T * H * dk and v.numel() == T * HV * dv):
        raise ValueError("gdn_prefill expects contiguous q, k [T, H*dk] and v [T, HV*dv]")
    LAUNCHES[0] += 1
    _lib.call("qw_gdn_prefill", q.data_ptr(), k.data_ptr(), v.data_ptr(), ba.data_ptr(), ba.stride(0),
              A_log.data_ptr(), dt_bias.data_ptr(), cu.data_ptr(), slots.data_ptr(), B, T, state.shape[0],
              state.data_ptr(), z.data_ptr(), z.stride(0), norm_w.data_ptr(), y.data_ptr(), y.stride(0), H, HV, dk,
              dv, scale, eps, _stream())


def gdn_decode(qkvz, ba, conv_w, conv_state, state, slots, B, A_log, dt_bias, norm_w, y, H, HV, dk, dv, eps):
    LAUNCHES[0] += 1
    _lib.call("qw_gdn_decode", qkvz.data_ptr(), qkvz.stride(0), ba.data_ptr(), ba.stride(0), conv_w.data_ptr(),
              conv_state.data_ptr(), state.data_ptr(), slots.data_ptr(), B, state.shape[0], A_log.data_ptr(),
              dt_bias.data_ptr(), norm_w.data_ptr(), y.data_ptr(), y.stride(0), H, HV, dk, dv, eps, _stream())


# ----------------------------------------------------------------------------- cache
def kv_grow(src_k, src_v, dst_k, dst_v, lengths, S, old_cap, new_cap):
    row_elems = src_k[0].numel()
    LAUNCHES[0] += 1
    _lib.call("qw_kv_grow", src_k.data_ptr(), src_v.data_ptr(), dst_k.data_ptr(), dst_v.data_ptr(),
              lengths.data_ptr(), S, old_cap, new_cap, row_elems, _stream())


KV_GROW_MAX_LAYERS = 32  # QW_KV_GROW_MAX_LAYERS


def kv_grow_layers(src, dst, lengths, S, old_cap, new_cap):
    """The growth of every layer's (K, V) pools (``src``, ``dst``: lists of (K, V) pairs of
    equal row size) in one launch per QW_KV_GROW_MAX_LAYERS layers."""
    import ctypes
    row_elems = src[0][0][0].numel()
    for i in range(0, len(src), KV_GROW_MAX_LAYERS):
        s_part, d_part = src[i:i + KV_GROW_MAX_LAYERS], dst[i:i + KV_GROW_MAX_LAYERS]
        n = len(s_part)
        arrs = [(ctypes.c_void_p * n)(*[t.data_ptr() for t in col]) for col in
                ([k for k, _ in s_part], [v for _, v in s_part], [k for k, _ in d_part], [v for _, v in d_part])]
        LAUNCHES[0] += 1
        _lib.call("qw_kv_grow_layers", *[ctypes.addressof(a) for a in arrs], n, lengths.data_ptr(), S, old_cap,
                  new_cap, row_elems, _stream())
