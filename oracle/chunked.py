"""The chunked (WY) form of the gated delta rule with bf16 operands inside each chunk, at
the rounding points of the prefill kernel (TEST INFRASTRUCTURE ONLY).

The reference computes prefill GDN with flashinfer's chunked kernel
(``chunk_gated_delta_rule``, reference/qwen38_inference.py:4852, 5084), which evaluates the
per-token recurrence of ``gdn_recurrence`` (oracle/ops.py; REF:1355-1408) in chunks of 64
tokens with bf16 tensor-core operands and fp32 accumulation. Rounding the operands changes
the output by about 1e-2 relative to the fp32 per-token recurrence, far more than one bf16
ulp, so a tight GPU parity bound needs a restatement that rounds where the kernel rounds.
This is that restatement of ``csrc/gdn_prefill.cu``:

* gating: g = -exp(A_log) softplus(a + dt_bias) (threshold 20), beta = bf16(sigmoid(b))
  (REF:1274-1289); G = cumulative sum of g within the chunk; decays e^{G_t - G_s} as
  2^{(G_t - G_s) log2 e};
* A_ts = beta_t e^{G_t-G_s} (k_t . k_s) for s < t, fp32; P_ts = bf16(scale e^{G_t-G_s} (q_t . k_s))
  for s <= t;
* T = (I + A)^-1 by 16 x 16 blocks: diagonal blocks by forward substitution in fp32, the
  blocks below by two levels of tf32 products (M_ik = T_ii A_ik, T_ij = -sum_k M_ik T_kj),
  then T rounded to bf16;
* bf16 tiles beta e^G K, e^{G_C-G} K and beta V; W = T (beta e^G K), stored as bf16(-W);
* per chunk: S0 = bf16(S); U = T (beta V) + (-W) S0^T rounded to bf16; O = bf16(scale e^G
  (Q S0^T) + P U); S = e^{G_C} S + U^T (e^{G_C-G} K), fp32.

Products of bf16 operands are accumulated in float64 and rounded to fp32 once (the kernel
accumulates in fp32 in its own order; the difference is a few fp32 ulps of each sum).
``tests/test_chunked_oracle_cpu.py`` checks this restatement against the per-token
recurrence; the GPU test of the prefill kernel compares against it in bf16 ulps.
"""
from __future__ import annotations

import torch

from .ops import bf16

_bf16 = bf16
F32, F64 = torch.float32, torch.float64
C = 64  # chunk length
LOG2E = 1.4426950408889634


def _ident(x):
    return x


def tf32(x: torch.Tensor) -> torch.Tensor:
    """cvt.rna.tf32.f32: fp32 to 10 mantissa bits, round to nearest with ties away from zero."""
    b = x.to(F32).contiguous().view(torch.int32)
    b = (b + 0x1000) & -0x2000
    return b.view(F32)


def _mm(a, b):
    """fp32 result of a product of (already rounded) operands, accumulated in float64."""
    return (a.to(F64) @ b.to(F64)).to(F32)


def _inverse_blocked(A, rtf=tf32):
    """(I + A)^-1 for strictly lower-triangular A [64, 64] fp32, as the kernel's blocked
    inverse: fp32 diagonal blocks, tf32 products for the blocks below."""
    T = torch.zeros(C, C, dtype=F32)
    diag = []
    for i in range(4):
        a = A[16 * i:16 * i + 16, 16 * i:16 * i + 16].to(F64)
        t = torch.zeros(16, 16, dtype=F64)
        for j in range(16):
            col = torch.zeros(16, dtype=F64)
            col[j] = 1.0
            for r in range(j + 1, 16):
                col[r] = -(a[r, :r] @ col[:r])
            t[:, j] = col
        diag.append(t.to(F32))
        T[16 * i:16 * i + 16, 16 * i:16 * i + 16] = diag[i]
    blk = lambda X, i, j: X[16 * i:16 * i + 16, 16 * j:16 * j + 16]  # noqa: E731
    M = {}
    for i in range(1, 4):
        for k in range(i):
            M[(i, k)] = _mm(rtf(diag[i]), rtf(blk(A, i, k)))
    Tij = {}
    for d in range(1, 4):
        for j in range(4 - d):
            i = j + d
            acc = torch.zeros(16, 16, dtype=F64)
            for k in range(j, i):
                rhs = diag[j] if k == j else Tij[(k, j)]
                acc += rtf(M[(i, k)]).to(F64) @ rtf(rhs).to(F64)
            Tij[(i, j)] = (-acc).to(F32)
            T[16 * i:16 * i + 16, 16 * j:16 * j + 16] = Tij[(i, j)]
    return T


def gating(a, b, A_log, dt_bias):
    """g (fp32 log decay) and beta (bf16-rounded) per token and value head: a, b [n, HV]."""
    x = a.to(F32) + dt_bias.to(F32)
    sp = torch.where(x <= 20.0, torch.log1p(torch.exp(x)), x)
    g = -torch.exp(A_log.to(F32)) * sp
    return g, bf16(torch.sigmoid(b.to(F32)))


def chunked_head(q, k, v, g, beta, S, scale, operand_rounding=True):
    """One value head. q, k [n, dk] and v [n, dv] bf16 values (as fp32); g, beta [n] fp32;
    S [dv, dk] fp32 initial state. Returns o [n, dv] (bf16 values) and the final state.
    ``operand_rounding=False`` keeps every intermediate in fp32 (the chunk algebra alone)."""
    bf16 = _bf16 if operand_rounding else _ident
    rtf = tf32 if operand_rounding else _ident
    n, dk = q.shape
    dv = v.shape[1]
    S = S.to(F32).clone()
    out = torch.empty(n, dv, dtype=F32)
    t_idx = torch.arange(C)
    lower = t_idx[:, None] > t_idx[None, :]
    causal = t_idx[:, None] >= t_idx[None, :]
    for c0 in range(0, n, C):
        m = min(C, n - c0)

        def pad(x):  # rows past the request are zero in the kernel's tiles
            return torch.cat([x[c0:c0 + m].to(F32), x.new_zeros((C - m,) + tuple(x.shape[1:])).to(F32)])

        Q, K, V, gg, bt = pad(q), pad(k), pad(v), pad(g), pad(beta)
        G = torch.cumsum(gg.to(F64), 0).to(F32)
        G2 = G * LOG2E
        dec = torch.exp2((G2[:, None] - G2[None, :]).to(F64)).to(F32)
        EGl, EG, EC = torch.exp(G[-1] - G), torch.exp(G), torch.exp(G[-1])
        KK, QK = _mm(K, K.T), _mm(Q, K.T)
        A = torch.where(lower, (bt[:, None] * dec) * KK, torch.zeros(()))
        P = bf16(torch.where(causal, (scale * dec) * QK, torch.zeros(())))
        Tb = bf16(_inverse_blocked(A, rtf))
        kb = bf16(K * (bt * EG)[:, None])
        kd = bf16(K * EGl[:, None])
        bv = bf16(V * bt[:, None])
        Wn = bf16(-_mm(Tb, kb))
        S0 = bf16(S)
        S = S * EC
        U = bf16(((Tb.to(F64) @ bv.to(F64)) + (Wn.to(F64) @ S0.T.to(F64))).to(F32))
        O1 = _mm(Q, S0.T)
        O2 = _mm(P, U)
        o = bf16(O1 * (scale * EG)[:, None] + O2)
        S = (S.to(F64) + U.T.to(F64) @ kd.to(F64)).to(F32)
        out[c0:c0 + m] = o[:m]
    return out, S


def chunked_gdn(q, k, v, a, b, A_log, dt_bias, state, scale, head_ratio, operand_rounding=True):
    """All value heads of one request: q, k [n, H, dk]; v [n, HV, dv]; a, b [n, HV] (the
    ba projection's columns); state [HV, dv, dk]. Returns o [n, HV, dv] and the state."""
    n, HV = v.shape[0], v.shape[1]
    g, beta = gating(a, b, A_log, dt_bias)
    o = torch.empty(n, HV, v.shape[2], dtype=F32)
    S = torch.empty_like(state, dtype=F32)
    for hv in range(HV):
        h = hv // head_ratio
        o[:, hv], S[hv] = chunked_head(q[:, h], k[:, h], v[:, hv], g[:, hv], beta[:, hv], state[hv], scale,
                                       operand_rounding)
    return o, S


__all__ = ["tf32", "gating", "chunked_head", "chunked_gdn", "C"]
