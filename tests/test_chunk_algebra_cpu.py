"""The chunked WY form of the gated delta rule, as the prefill kernel computes it
(csrc/gdn_prefill.cu: chunks of 64 tokens, partial chunks zero-padded, the state products
transposed with the value dimension first), in float64 against the oracle's
token-by-token recurrence (oracle/ops.py gdn_recurrence, REF:1355-1408).

This pins the chunk algebra on the CPU: the WY inverse, the decay bookkeeping, the
transposed U^T / O^T products and the carried state. The GPU tests pin the kernel's
arithmetic to the same oracle. Tolerance: 1e-4 absolute + 1e-4 relative (the oracle runs in
float32).
"""
import pytest
import torch

from oracle.ops import gdn_recurrence

C = 64  # chunk length of the kernel
F64 = torch.float64


def chunked_head(q, k, v, g, beta, S0, scale):
    """One value head. q, k: [n, dk]; v: [n, dv]; g, beta: [n]; S0: [dv, dk]. Returns
    o [n, dv] and the final state [dv, dk]."""
    n = q.shape[0]
    S = S0.clone()
    out = torch.empty(n, v.shape[1], dtype=F64)
    lower = torch.tril(torch.ones(C, C, dtype=torch.bool), -1)
    causal = torch.tril(torch.ones(C, C, dtype=torch.bool))
    for c0 in range(0, n, C):
        m = min(C, n - c0)

        def pad(x):  # rows past the request are zero, as the kernel's cleared tile rows
            return torch.cat([x[c0:c0 + m], x.new_zeros((C - m,) + tuple(x.shape[1:]))])

        Q, K, V, gg, b = pad(q), pad(k), pad(v), pad(g), pad(beta)
        G = torch.cumsum(gg, 0)
        Dec = torch.exp(G[:, None] - G[None, :])  # e^{G_t - G_s}
        A = torch.where(lower, b[:, None] * Dec * (K @ K.T), 0.0)
        T = torch.linalg.inv(torch.eye(C, dtype=F64) + A)
        W = T @ ((b * torch.exp(G))[:, None] * K)  # T diag(b e^G) K
        Ut = (b[:, None] * V).T @ T.T + S @ (-W).T  # U^T = (bV)^T T^T + S0 (-W)^T
        P = torch.where(causal, scale * Dec * (Q @ K.T), 0.0)
        Ot = scale * (S @ Q.T) * torch.exp(G)[None, :] + Ut @ P.T  # O1^T scaled + O2^T
        S = torch.exp(G[-1]) * S + Ut @ (torch.exp(G[-1] - G)[:, None] * K)
        out[c0:c0 + m] = Ot.T[:m]
    return out, S


@pytest.mark.parametrize("n", [1, 63, 64, 65, 130, 200])
def test_chunked_form_matches_token_recurrence(n):
    gen = torch.Generator().manual_seed(100 + n)
    H, HV, dk, dv = 1, 2, 32, 32
    scale = dk ** -0.5
    q = torch.nn.functional.normalize(torch.randn(n, H, dk, generator=gen, dtype=F64), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(n, H, dk, generator=gen, dtype=F64), dim=-1)
    v = torch.randn(n, HV, dv, generator=gen, dtype=F64)
    g = -0.5 * torch.nn.functional.softplus(torch.randn(n, HV, generator=gen, dtype=F64))
    beta = torch.sigmoid(torch.randn(n, HV, generator=gen, dtype=F64))
    S0 = 0.1 * torch.randn(HV, dv, dk, generator=gen, dtype=F64)

    o_ref, S_ref = gdn_recurrence(q.float(), k.float(), v.float(), g.float(), beta.float(), S0.float(), scale,
                                  HV // H)
    for hv in range(HV):
        o, S = chunked_head(q[:, hv // (HV // H)], k[:, hv // (HV // H)], v[:, hv], g[:, hv], beta[:, hv], S0[hv],
                            scale)
        torch.testing.assert_close(o, o_ref[:, hv].double(), atol=1e-4, rtol=1e-4)
        torch.testing.assert_close(S, S_ref[hv].double(), atol=1e-4, rtol=1e-4)
