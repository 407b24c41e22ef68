"""Per-op CPU restatements of the reference arithmetic (TEST INFRASTRUCTURE ONLY).

Every function computes in fp32 and applies ``rnd`` exactly where the reference rounds to
its storage dtype (bf16 in the 27B model). ``rnd`` is :func:`bf16` for the bf16-faithful
mode and :func:`ident` for the fp32 tiny configuration. Citations are
``reference/qwen38_inference.py`` line numbers ("REF").
"""
from __future__ import annotations

import math

import torch

F32 = torch.float32


def bf16(x: torch.Tensor) -> torch.Tensor:
    """Round to bfloat16 (round-to-nearest-even) and widen back to fp32."""
    return x.to(torch.bfloat16).to(F32)


def ident(x: torch.Tensor) -> torch.Tensor:
    return x


def f32(x: torch.Tensor) -> torch.Tensor:
    return x.to(F32)


# ----------------------------------------------------------------------------- norms
def gemma_rmsnorm(x, w, eps, rnd):
    """sgl_kernel ``gemma_rmsnorm`` (REF:4851, call REF:5050): x*rsqrt(mean x^2+eps)*(1+w)."""
    x = f32(x)
    r = torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return rnd(x * r * (1.0 + f32(w)))


def gemma_add_rmsnorm(x, residual, w, eps, rnd):
    """sgl_kernel ``gemma_fused_add_rmsnorm`` (REF:4851, calls REF:5052/5088/5093).

    h = x + residual in fp32; residual <- rnd(h); x <- rnd(norm(h)) using the unrounded h.
    Returns ``(x_new, residual_new)``.
    """
    h = f32(x) + f32(residual)
    r = torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    return rnd(h * r * (1.0 + f32(w))), rnd(h)


def gated_rmsnorm(x, w, z, eps, rnd):
    """``_layer_norm_fwd_1pass_kernel`` in RMS mode with norm_before_gate=True
    (REF:1836-1926): y = x*rsqrt(mean x^2+eps)*w * z*sigmoid(z); plain w (no +1)."""
    x = f32(x)
    var = x.pow(2).mean(-1, keepdim=True)
    y = x * torch.rsqrt(var + eps) * f32(w)
    z = f32(z)
    return rnd(y * (z * torch.sigmoid(z)))


def l2norm(x, eps=1e-6):
    """``l2norm_fwd_kernel`` (REF:1583-1589): x / sqrt(sum x^2 + eps), fp32."""
    x = f32(x)
    return x / torch.sqrt(x.pow(2).sum(-1, keepdim=True) + eps)


# ----------------------------------------------------------------------------- dense
def linear(x, w, rnd):
    """``F.linear`` (REF:5054 etc.): fp32 accumulate of storage-dtype operands, rounded.
    Weights of more than 2^26 elements (the 27B lm_head) are widened 2^15 rows at a time,
    so the fp32 copy stays small; each output is the same K-long dot product either way."""
    if w.numel() <= 1 << 26:
        return rnd(f32(x) @ f32(w).t())
    xf = f32(x)
    return rnd(torch.cat([xf @ f32(w[i:i + 32768]).t() for i in range(0, w.shape[0], 32768)], dim=-1))


def silu_mul(gate_up, rnd):
    """SGLang ``act_and_mul_kernel<kSiLU>`` (REF:2238-2281): rnd(silu(g) * u) in fp32."""
    gu = f32(gate_up)
    n = gu.shape[-1] // 2
    g, u = gu[..., :n], gu[..., n:]
    return rnd(g / (1.0 + torch.exp(-g)) * u)


# ----------------------------------------------------------------------------- attention
def qk_norm_rope_gate(qg, k, q_w, k_w, rope, positions, eps, nq, nkv, d, rd, rnd):
    """``_fused_qk_rmsnorm_rope_gate_kernel`` (REF:116-184).

    qg: [T, nq*2*d] (per head [q | gate]); k: [T, nkv*d]. Returns q [T,nq,d], k [T,nkv,d],
    gate [T,nq,d]. Gemma norm of each head (rounded), NeoX rotate-half RoPE on the first
    ``rd`` dims with the fp32 [cos | sin] table, pass-through tail carries the rounded norm.
    """
    T = qg.shape[0]
    qg = f32(qg).view(T, nq, 2 * d)
    q_in, gate = qg[..., :d], qg[..., d:]
    k_in = f32(k).view(T, nkv, d)

    def one(x, w):
        inv = torch.rsqrt(x.pow(2).sum(-1, keepdim=True) / d + eps)
        xn = rnd(x * inv * (f32(w) + 1.0))
        half = rd // 2
        cs = rope[positions.long()]  # [T, rd]
        cos = cs[:, None, :half]
        sin = cs[:, None, half:rd]
        x1, x2 = xn[..., :half], xn[..., half:rd]
        out = xn.clone()
        out[..., :half] = rnd(x1 * cos - x2 * sin)
        out[..., half:rd] = rnd(x2 * cos + x1 * sin)
        return out

    return one(q_in, q_w), one(k_in, k_w), gate.clone()


def sigmoid_mul(attn, gate, rnd):
    """``_fused_sigmoid_mul_kernel`` (REF:2105-2121): rnd(attn * sigmoid(gate))."""
    return rnd(f32(attn) * torch.sigmoid(f32(gate)))


def paged_attention(q, kc, vc, starts, prefixes, lens, scale, rnd):
    """Causal varlen GQA attention over the slot-contiguous KV rows (the math of the
    trtllm-gen context/decode kernels, REF:5059-5064).

    q: [T, nq, d] (roped); kc/vc: [rows, nkv, d]; ``starts[i]`` = first cache row of request
    i; query j of request i (position prefixes[i]+j) sees keys 0..prefixes[i]+j.
    """
    T, nq, d = q.shape
    nkv = kc.shape[1]
    grp = nq // nkv
    out = torch.empty(T, nq, d, dtype=F32)
    t0 = 0
    for s0, p, n in zip(starts, prefixes, lens):
        L = p + n
        K = f32(kc[s0:s0 + L]).repeat_interleave(grp, dim=1)  # [L, nq, d]
        V = f32(vc[s0:s0 + L]).repeat_interleave(grp, dim=1)
        Q = f32(q[t0:t0 + n])  # [n, nq, d]
        S = torch.einsum("tnd,lnd->ntl", Q, K) * scale  # [nq, n, L]
        qpos = p + torch.arange(n)
        mask = torch.arange(L)[None, :] > qpos[:, None]
        S = S.masked_fill(mask[None], float("-inf"))
        P = torch.softmax(S, dim=-1)
        out[t0:t0 + n] = torch.einsum("ntl,lnd->tnd", P, V)
        t0 += n
    return rnd(out)


# ----------------------------------------------------------------------------- GDN
def conv_prefill(x, w, conv_state, cu, slots, has_initial, rnd):
    """``_causal_conv1d_fwd_kernel`` (REF:750-1076) + its state update (REF:857-963).

    x: [T, C] (storage-dtype values); w: [C, W]; conv_state: [S, C, W-1] updated in place.
    Per channel: acc = sum_j rnd(x[t-W+1+j]*w[j]) over taps j=0..W-1 in order (products of
    two storage-dtype values are rounded to that dtype, REF:1052), then silu, rounded.
    History before the first token comes from conv_state[slot] if has_initial else zeros.
    """
    x = f32(x)
    w = f32(w)
    T, C = x.shape
    W = w.shape[1]
    sl = W - 1
    out = torch.empty(T, C, dtype=F32)
    for i in range(len(cu) - 1):
        a, b = cu[i], cu[i + 1]
        n = b - a
        s = slots[i]
        hist = f32(conv_state[s]).t().clone() if has_initial[i] else torch.zeros(sl, C)
        seq = torch.cat([hist, x[a:b]], 0)  # [sl+n, C]
        acc = torch.zeros(n, C)
        for j in range(W):
            acc = acc + rnd(seq[j:j + n] * w[:, j])
        out[a:b] = rnd(acc / (1.0 + torch.exp(-acc)))
        # state <- last W-1 raw inputs of [history, x] (zeros before x when no history)
        conv_state[s] = seq[-sl:].t().to(conv_state.dtype)
    return out


def conv_decode(x, w, conv_state, slots, rnd):
    """``_fused_qkvzba_causal_conv1d_update_contiguous_kernel`` (REF:334-414).

    x: [B, C]; acc = sum_{p<W-1} rnd(state[p]*w[p]) + rnd(x*w[W-1]); silu; state shifts
    left and appends the raw x. A slot outside [0, S) leaves the output = x (REF:349-391).
    """
    x = f32(x)
    w = f32(w)
    B, C = x.shape
    W = w.shape[1]
    out = torch.empty(B, C, dtype=F32)
    for i in range(B):
        s = slots[i]
        if not (0 <= s < conv_state.shape[0]):
            out[i] = x[i]
            continue
        st = f32(conv_state[s])  # [C, W-1]
        acc = torch.zeros(C)
        for p in range(W - 1):
            acc = acc + rnd(st[:, p] * w[:, p])
        acc = acc + rnd(x[i] * w[:, W - 1])
        out[i] = acc / (1.0 + torch.exp(-acc))
        conv_state[s] = torch.cat([st[:, 1:], x[i][:, None]], 1).to(conv_state.dtype)
    return rnd(out)


def gdn_gating(A_log, a, b, dt_bias, rnd):
    """``fused_gdn_gating_kernel`` (REF:1274-1289): g = -exp(A_log)*softplus(a+dt_bias)
    (threshold 20, beta 1), fp32; beta = rnd(sigmoid(b)) stored fp32."""
    x = f32(a) + f32(dt_bias)
    sp = torch.where(x <= 20.0, torch.log(1.0 + torch.exp(x)), x)
    g = -torch.exp(f32(A_log)) * sp
    beta = rnd(torch.sigmoid(f32(b)))
    return g, beta


def gdn_recurrence(q, k, v, g, beta, state, scale, head_ratio):
    """The gated delta rule, token by token (the decode kernel REF:1355-1408 applied per
    token; flashinfer's chunked prefill computes the same recurrence in chunks).

    q,k: [n, H, dk]; v: [n, HV, dv]; g, beta: [n, HV] (g = log decay); state: [HV, dv, dk]
    fp32, updated and returned. Per token: S *= exp(g); v' = beta*(v - S k);
    S += v' k^T; o = S (q*scale). Returns o [n, HV, dv] fp32.
    """
    n = q.shape[0]
    HV = v.shape[1]
    hidx = torch.arange(HV) // head_ratio
    S = state.clone()
    out = torch.empty(n, HV, v.shape[2], dtype=F32)
    for t in range(n):
        qt = f32(q[t])[hidx] * scale  # [HV, dk]
        kt = f32(k[t])[hidx]
        vt = f32(v[t])
        S = S * torch.exp(g[t])[:, None, None]
        vp = (vt - torch.einsum("hvk,hk->hv", S, kt)) * beta[t][:, None]
        S = S + vp[:, :, None] * kt[:, None, :]
        out[t] = torch.einsum("hvk,hk->hv", S, qt)
    return out, S
