"""The online softmax of the prefill attention kernel and the split merge of the split-KV
kernels (csrc/attention.cu), restated in float64 with the kernel's bf16 rounding of P,
against exact softmax attention. The GPU tests pin the kernels themselves to the oracle.

The kernel's online softmax works in the log2 domain over blocks of 64 keys. The running
max of a row is raised only when a block's max exceeds it by more than 8, and then O and l
are rescaled. Weights are 2^(s scale log2 e - m) and can reach 2^8; they are rounded to
bf16 for the P V product and summed in fp32 for l. Splits over the keys return
(m, l, unnormalised O). The merge weights each split by 2^(m_s - max m); a split with no
keys (m = -inf) gets weight 0. Tolerance: 4e-3 relative to the largest |output|, about
two bf16 ulps of P.
"""
import math

import pytest
import torch

BLK = 64
LOG2E = 1.4426950408889634


def bf16(x):
    return x.to(torch.bfloat16).to(torch.float64)


def online_split(s, v, scale):
    """One split: scores s [n] of one query row, values v [n, d]. Returns (m, l, o)."""
    m, l = -math.inf, 0.0
    o = torch.zeros(v.shape[1], dtype=torch.float64)
    sl2 = scale * LOG2E
    for j0 in range(0, s.shape[0], BLK):
        blk = s[j0:j0 + BLK]
        mx = sl2 * float(blk.max())
        if mx > m + 8.0:  # raise the running max (and rescale what is accumulated)
            if m != -math.inf:
                alpha = 2.0 ** (m - mx)
                o = o * alpha
                l = l * alpha
            m = mx
        p = torch.exp2(blk * sl2 - m)
        l += float(p.sum())
        o = o + bf16(p) @ v[j0:j0 + BLK]
    return m, l, o


def merge(parts):
    mm = max(m for m, _, _ in parts)
    ll = sum(l * (0.0 if m == -math.inf else 2.0 ** (m - mm)) for m, l, _ in parts)
    oo = sum(o * (0.0 if m == -math.inf else 2.0 ** (m - mm)) for m, _, o in parts)
    return oo / ll


@pytest.mark.parametrize("n,splits", [(64, 1), (200, 1), (1000, 1), (1000, 4), (777, 7), (130, 3)])
def test_online_softmax_and_split_merge(n, splits):
    g = torch.Generator().manual_seed(n * 10 + splits)
    d, scale = 64, 64 ** -0.5
    # scores that grow along the keys, so later blocks raise the running max several times
    s = torch.randn(n, generator=g, dtype=torch.float64) * (1.0 + 0.2 * torch.arange(n, dtype=torch.float64))
    v = torch.randn(n, d, generator=g, dtype=torch.float64)
    exact = torch.softmax(s * scale, 0) @ v
    per = -(-n // splits)
    parts = []
    for i in range(splits + 1):  # one split more than needed: it holds no keys (m = -inf)
        lo, hi = i * per, min(n, (i + 1) * per)
        parts.append(online_split(s[lo:hi], v[lo:hi], scale) if lo < hi
                     else (-math.inf, 0.0, torch.zeros(d, dtype=torch.float64)))
    got = merge(parts)
    assert float((got - exact).abs().max()) <= 4e-3 * float(exact.abs().max())


def test_threshold_keeps_weights_bounded():
    """With the lazy raise no weight exceeds 2^8 (fp32 and bf16 stay far from overflow)."""
    s = torch.linspace(0.0, 400.0, 1024, dtype=torch.float64)
    m, sl2 = -math.inf, LOG2E
    top = 0.0
    for j0 in range(0, 1024, BLK):
        mx = sl2 * float(s[j0:j0 + BLK].max())
        if mx > m + 8.0:
            m = mx
        top = max(top, float(torch.exp2(s[j0:j0 + BLK] * sl2 - m).max()))
    assert top <= 2.0 ** 8
