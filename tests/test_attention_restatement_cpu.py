"""The CPU restatement of the attention kernels' arithmetic (oracle/attention_kernels.py)
against the math of the reference's attention (oracle.ops.paged_attention, then the sigmoid
gate), CPU only: they differ only by where P is rounded to bf16 and by the order of fp32
sums, so they agree within the bound the GPU tests use against the math oracle (4 bf16
ulps plus 2e-3), and the lazily raised running maximum of the prefill kernel is exercised
(keys whose magnitude grows with position)."""
import pytest
import torch

from oracle import ops as O
from oracle import attention_kernels as AK


def _case(seed, nq, nkv, d, prefixes, lens, cap, grow=False):
    g = torch.Generator().manual_seed(seed)
    S = len(lens)
    rows = S * cap + 64
    kc = O.bf16(torch.randn(rows, nkv, d, generator=g))
    vc = O.bf16(torch.randn(rows, nkv, d, generator=g))
    if grow:
        pos = torch.arange(rows, dtype=torch.float32).view(-1, 1, 1)
        kc = O.bf16(kc * (1.0 + pos / 64.0))
    T = sum(lens)
    qkv = O.bf16(torch.randn(T, 2 * nq * d + 2 * nkv * d, generator=g))
    starts = [64 + s * cap for s in range(S)]
    return kc, vc, qkv, starts


def _math(qkv, nq, d, kc, vc, starts, prefixes, lens, scale):
    T = qkv.shape[0]
    q = qkv[:, :2 * nq * d].view(T, nq, 2 * d)
    att = O.paged_attention(q[..., :d], kc, vc, starts, prefixes, lens, scale, O.bf16)
    return O.sigmoid_mul(att.reshape(T, -1), q[..., d:].reshape(T, -1), O.bf16)


def _close(got, exp, n_ulp, atol, max_frac):
    d = (got - exp).abs()
    ulp = torch.exp2(torch.floor(torch.log2(torch.maximum(got.abs(), exp.abs()).clamp_min(2.0 ** -126))) - 7)
    assert bool((d <= n_ulp * ulp + atol).all()), f"max diff {d.max().item():.3g}"
    assert (d > 0).float().mean().item() <= max_frac


@pytest.mark.parametrize("grow", [False, True])
def test_prefill_restatement_matches_math(grow):
    nq, nkv, d = 4, 2, 64
    prefixes, lens = ([0, 37, 130], [70, 1, 77]) if not grow else ([0, 100], [200, 60])
    kc, vc, qkv, starts = _case(3, nq, nkv, d, prefixes, lens, cap=512, grow=grow)
    scale = d ** -0.5
    got = AK.attn_prefill(qkv, nq, nkv, d, kc, vc, starts, prefixes, lens, scale)
    exp = _math(qkv, nq, d, kc, vc, starts, prefixes, lens, scale)
    _close(got, exp, 4, 2e-3 if not grow else 1.6e-2, 0.5)


@pytest.mark.parametrize("splits", [1, 3])
def test_decode_restatement_matches_math(splits):
    nq, nkv, d = 4, 2, 64
    prefixes = [1, 63, 64, 300, 511]
    lens = [1] * len(prefixes)
    kc, vc, qkv, starts = _case(5, nq, nkv, d, prefixes, lens, cap=512)
    scale = d ** -0.5
    got = AK.attn_decode(qkv, nq, nkv, d, kc, vc, starts, [p + 1 for p in prefixes], 512, splits, scale)
    exp = _math(qkv, nq, d, kc, vc, starts, prefixes, lens, scale)
    _close(got, exp, 4, 2e-3, 0.5)
