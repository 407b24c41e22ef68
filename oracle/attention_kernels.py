"""The attention kernels' own arithmetic, restated on the CPU (TEST INFRASTRUCTURE ONLY).

The reference computes attention with trtllm-gen's context and decode kernels
(reference/qwen38_inference.py:5059-5064), whose internal rounding is not published;
``oracle.ops.paged_attention`` states the math (softmax(Q K^T) V in fp32, rounded once).
A kernel that feeds P to the tensor cores rounds it to bf16 first, and where it does so
depends on its running maximum, so against that oracle an output can move by several bf16
ulps. These functions repeat the steps of ``csrc/attention.cu`` in fp32 so that the GPU
tests can bound the kernels at the level of one ulp:

* prefill (``attn_prefill_kernel``): keys in blocks of 64; per row the block maximum of the
  raw scores s, scaled by scale * log2(e); the running maximum m is raised to it only when
  it exceeds m by more than 8 (then O and l are multiplied by 2^(m_old - m_new));
  p = 2^(s * scale log2 e - m) in fp32, l += sum(p), O += bf16(p) V; at the end
  out = bf16(bf16(O (1 / l)) / (1 + e^-gate));
* decode (``attn_decode_kernel`` + ``attn_decode_combine_kernel``): the keys of a request
  split into ranges of ``kps`` keys, each range into two halves of 16-key steps (one per
  warp); per step an exact running maximum (O and l scaled by 2^(m_old - m_new) every step),
  p = 2^(s * scale log2 e - m), O += bf16(p) V; the two halves and then the ranges are merged
  with weights 2^(m_i - max m) in fp32; out = bf16(bf16(O / l) / (1 + e^-gate)).

Dot products are formed in float64 and rounded to fp32 once (the kernels accumulate on the
tensor cores in fp32 in their own order: a few fp32 ulps of each sum); 2^x uses the exact
function where the kernels use the hardware approximation (two ulps). Those differences
move a bf16 output only when it sits next to a rounding boundary.
"""
from __future__ import annotations

import math

import torch

F32, F64 = torch.float32, torch.float64
LOG2E = 1.4426950408889634


def _bf16(x):
    return x.to(torch.bfloat16).to(F32)


def _dot(a, b):
    """a [n, d] @ b [m, d]^T of bf16-valued fp32 tensors: float64 sums rounded to fp32."""
    return (a.to(F64) @ b.to(F64).t()).to(F32)


def _fma_f32(a, b, c):
    """fp32 a * b + c with one rounding (the float64 product of two fp32 values is exact)."""
    return (a.to(F64) * b + c.to(F64)).to(F32)


def _gate(a, gate):
    return _bf16(a / (1.0 + torch.exp(-gate)))


def attn_prefill_head(q, k, v, gate, prefix, scale, block=64, lazy=8.0):
    """One query head of one request through the prefill kernel's steps.

    q, gate: [n, d] (bf16 values, roped q); k, v: [prefix + n, d] (the request's cache rows for
    this head's KV head). Query j sits at position prefix + j and sees keys 0 .. prefix + j.
    Returns [n, d] fp32 holding bf16 values."""
    n, d = q.shape
    L = k.shape[0]
    sl2 = torch.tensor(scale * LOG2E, dtype=F32)
    m = torch.full((n,), float("-inf"), dtype=F32)
    l = torch.zeros(n, dtype=F32)
    o = torch.zeros(n, d, dtype=F32)
    qpos = prefix + torch.arange(n)
    for j, k0 in enumerate(range(0, L, block)):
        kb, vb = k[k0:k0 + block], v[k0:k0 + block]
        s = _dot(q, kb)  # [n, b]
        keys = k0 + torch.arange(kb.shape[0])
        s = s.masked_fill(keys[None, :] > qpos[:, None], float("-inf"))
        mx = sl2 * s.max(dim=1).values
        grow = mx > m + lazy
        m_new = torch.where(grow, mx, m)
        if j > 0:
            alpha = torch.where(grow, torch.exp2(m - m_new), torch.ones_like(m))
            o = o * alpha[:, None]
            l = l * alpha
        m = m_new
        mu = torch.where(torch.isinf(m) & (m < 0), torch.zeros_like(m), m)
        p = torch.exp2(_fma_f32(s, sl2, -mu[:, None]))
        l = l + p.sum(dim=1, dtype=F32)
        o = o + _dot(_bf16(p), vb.t().contiguous())
    inv_l = torch.where(l > 0, 1.0 / l, torch.zeros_like(l))
    return _gate(_bf16(o * inv_l[:, None]), gate)


def attn_prefill(qkv, nq, nkv, d, kc, vc, starts, prefixes, lens, scale):
    """All heads and requests: qkv [T, 2 nq d + ...] with q and gate interleaved per head;
    kc, vc [rows, nkv, d]. Returns [T, nq d]."""
    T = qkv.shape[0]
    grp = nq // nkv
    out = torch.empty(T, nq * d, dtype=F32)
    t0 = 0
    for s0, p, n in zip(starts, prefixes, lens):
        for h in range(nq):
            q = qkv[t0:t0 + n, h * 2 * d:h * 2 * d + d].to(F32)
            g = qkv[t0:t0 + n, h * 2 * d + d:(h + 1) * 2 * d].to(F32)
            kv = h // grp
            k = kc[s0:s0 + p + n, kv].to(F32)
            v = vc[s0:s0 + p + n, kv].to(F32)
            out[t0:t0 + n, h * d:(h + 1) * d] = attn_prefill_head(q, k, v, g, p, scale)
        t0 += n
    return out


def attn_decode_head(q, k, v, gate, kps, scale, warps=2, step=16):
    """One query head of one decode token through the decode kernel's steps: q, gate [d];
    k, v [L, d] (all keys of the request). kps = keys per split (the launcher's rounding of
    max_len / splits up to a multiple of 32). Returns [d]."""
    L, d = k.shape
    sl2 = torch.tensor(scale * LOG2E, dtype=F32)
    parts = []
    for k_begin in range(0, L, kps):
        k_end = min(L, k_begin + kps)
        span = -(-kps // (warps * step)) * step
        wparts = []
        for w in range(warps):
            w_begin = k_begin + w * span
            w_end = min(k_end, w_begin + span)
            m = torch.tensor(float("-inf"), dtype=F32)
            l = torch.tensor(0.0, dtype=F32)
            o = torch.zeros(d, dtype=F32)
            for key0 in range(w_begin, w_end, step):
                kb, vb = k[key0:min(w_end, key0 + step)], v[key0:min(w_end, key0 + step)]
                x = _dot(q[None], kb)[0] * sl2
                mn = torch.maximum(m, x.max())
                alpha = torch.exp2(m - mn)
                p = torch.exp2(x - mn)
                l = l * alpha + p.sum(dtype=F32)
                m = mn
                o = o * alpha + _dot(_bf16(p)[None], vb.t().contiguous())[0]
            wparts.append((m, l, o))
        parts.append(_merge(wparts))
    mm, ll, oo = _merge(parts)
    a = _bf16(torch.where(ll > 0, oo / ll, torch.zeros_like(oo)))
    return _gate(a, gate)


def _merge(parts):
    """(max, sum, O) partials merged with weights 2^(m_i - max m), in order, in fp32."""
    mm = max((float(m) for m, _, _ in parts), default=float("-inf"))
    mm = torch.tensor(mm, dtype=F32)
    ll = torch.tensor(0.0, dtype=F32)
    oo = torch.zeros_like(parts[0][2])
    for m, l, o in parts:
        f = torch.tensor(0.0, dtype=F32) if math.isinf(float(m)) and float(m) < 0 else torch.exp2(m - mm)
        ll = ll + l * f
        oo = oo + o * f
    return mm, ll, oo


def attn_decode(qkv, nq, nkv, d, kc, vc, starts, seq_lens, max_len, splits, scale):
    """All requests (one token each) and heads; the launcher's keys per split:
    kps = ceil(ceil(max_len / splits) / 32) * 32. Returns [B, nq d]."""
    B = qkv.shape[0]
    grp = nq // nkv
    kps = -(-(-(-max_len // splits)) // 32) * 32
    out = torch.empty(B, nq * d, dtype=F32)
    for b in range(B):
        L = seq_lens[b]
        for h in range(nq):
            q = qkv[b, h * 2 * d:h * 2 * d + d].to(F32)
            g = qkv[b, h * 2 * d + d:(h + 1) * 2 * d].to(F32)
            kv = h // grp
            out[b, h * d:(h + 1) * d] = attn_decode_head(q, kc[starts[b]:starts[b] + L, kv].to(F32),
                                                         vc[starts[b]:starts[b] + L, kv].to(F32), g, kps, scale)
    return out
