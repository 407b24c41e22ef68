"""How far two correct implementations of the reference's arithmetic fall apart at the
logits (CPU only): the oracle with its GEMMs accumulated in fp32 against the same oracle
accumulating them in fp64, every bf16 rounding point unchanged.

The logits are float(bf16(h W^T)) (REF:5096), so a difference in an fp32 sum flips a bf16
rounding, and flips spread through the norms and projections of the following layers. This
measures the floor that the reference harness's atol = rtol = 1e-3 (test_forward_step.py:
122-134) leaves to any implementation that does not reproduce the reference's exact summation
order. Measured on the 27B width with 4 layers and the full vocabulary (QW_SLOW_TESTS=1, about
2 minutes): 24-28 % of logits within 1e-3, |d| up to 0.063, over prompts [7, 3] and two decode
steps; the mini width is the default case.
"""
import dataclasses
import os

import pytest
import torch

from oracle import OracleModel
from oracle import ops as O
from qwen38_inference_b200.config import mini, qwen38_27b, random_weights


def _linear_f64(x, w, rnd):
    if w.numel() <= 1 << 26:
        return rnd((x.double() @ w.double().t()).float())
    xd = x.double()
    return rnd(torch.cat([(xd @ w[i:i + 32768].double().t()).float() for i in range(0, w.shape[0], 32768)], -1))


def _agreement(cfg, monkeypatch, n_decode=2):
    w = random_weights(cfg, seed=7)
    ref = OracleModel(cfg, w, max_context=512)
    g = torch.Generator().manual_seed(0)
    ids = lambda n: torch.randint(cfg.vocab_size, (n,), generator=g).tolist()  # noqa: E731
    steps = [[ids(7), ids(3)]] + [[ids(1), ids(1)] for _ in range(n_decode)]

    def run():
        c = ref.new_cache(2, initial_capacity=64)
        return [ref.forward_step(s, c) for s in steps]
    a = run()
    with monkeypatch.context() as m:
        m.setattr(O, "linear", _linear_f64)
        b = run()
    out = []
    for x, y in zip(a, b):
        d = (x - y).abs()
        out.append(((d <= 1e-3 + 1e-3 * y.abs()).float().mean().item(), d.max().item()))
    return out


def test_summation_order_alone_breaks_the_strict_bound_mini(monkeypatch):
    res = _agreement(mini(num_layers=4, vocab=2048), monkeypatch)
    print("mini: fraction within 1e-3, max |d| per call:", res)
    # the two oracles stay within rounding-level distance of each other
    assert all(mx < 0.05 for _, mx in res)


@pytest.mark.skipif(os.environ.get("QW_SLOW_TESTS") != "1", reason="27B width: set QW_SLOW_TESTS=1 (~2 minutes)")
def test_summation_order_alone_breaks_the_strict_bound_27b_width(monkeypatch):
    torch.set_num_threads(max(1, len(os.sched_getaffinity(0))))
    res = _agreement(dataclasses.replace(qwen38_27b(), num_hidden_layers=4), monkeypatch)
    print("27B width: fraction within 1e-3, max |d| per call:", res)
    assert all(f < 0.5 for f, _ in res) and all(mx < 0.15 for _, mx in res)
