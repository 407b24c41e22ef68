"""Pin the CPU oracle against golden vectors from the reference's own Triton kernels.

The fixtures in tests/golden/ were produced by tests/golden/make_golden.py, which runs
reference/qwen38_inference.py's kernels under the (bf16-corrected) Triton CPU interpreter.
Tolerance: bf16 outputs may differ by at most one bf16 ulp, on at most 2% of elements
(summation order and fp32 transcendental rounding differ between numpy and torch); fp32
outputs within rtol 2e-5 / atol 1e-6. Pure copies and state shifts must be bit-exact.
"""
from pathlib import Path

import pytest
import torch

from oracle import ops

G = Path(__file__).parent / "golden"


def load(name):
    return torch.load(G / f"{name}.pt", weights_only=False)


def ulp_bf16(x):
    x = x.float().abs().clamp_min(2.0 ** -126)
    return torch.exp2(torch.floor(torch.log2(x)) - 7)


def assert_bf16_close(got, exp, max_frac=0.02):
    got, exp = got.float(), exp.float()
    diff = (got - exp).abs()
    tol = torch.maximum(ulp_bf16(exp), ulp_bf16(got)) * 1.01
    assert bool((diff <= tol).all()), f"max diff {diff.max().item()} beyond one bf16 ulp"
    frac = (diff > 0).float().mean().item()
    assert frac <= max_frac, f"{frac:.4f} of elements differ"


@pytest.mark.parametrize("tag", ["27b", "tiny"])
def test_qk_norm_rope_gate(tag):
    d = load(f"rope_{tag}")
    nq, nkv, hd, rd = d["nq"], d["nkv"], d["d"], d["rd"]
    qg, k, _ = d["qkv"].float().split([2 * nq * hd, nkv * hd, nkv * hd], dim=-1)
    q, kk, gate = ops.qk_norm_rope_gate(qg, k, d["q_w"], d["k_w"], d["rope"], d["positions"], 1e-6,
                                        nq, nkv, hd, rd, ops.bf16)
    assert_bf16_close(q.reshape(q.shape[0], -1), d["q"])
    assert_bf16_close(kk.reshape(kk.shape[0], -1), d["k"])
    assert torch.equal(gate.to(torch.bfloat16), d["gate"])


def test_conv_decode():
    d = load("conv_decode")
    st = d["state_in"].clone()
    C = d["C"]
    mixed = ops.conv_decode(d["qkvz"][:, :C], d["weight"], st, d["slots"].tolist(), ops.bf16)
    assert_bf16_close(mixed, d["mixed"])
    assert torch.equal(st, d["state_out"])  # shift + append is a pure copy
    assert torch.equal(d["qkvz"][:, C:].reshape(d["z"].shape), d["z"])


def test_conv_prefill_and_state():
    d = load("conv_prefill")
    st = d["state_in"].clone()
    C = d["C"]
    cu = d["cu"].tolist()
    y = ops.conv_prefill(d["x"][:, :C], d["weight"], st, cu, d["slots"], d["has_initial"], ops.bf16)
    assert_bf16_close(y, d["out"])
    assert torch.equal(st, d["state_out"])
    # the split kernel is a pure copy of the conv output
    assert torch.equal(d["out"][:, :128], d["q"].reshape(-1, 128))
    assert torch.equal(d["out"][:, 256:], d["v"].reshape(-1, 256))


def test_l2norm():
    d = load("l2norm")
    assert_bf16_close(ops.bf16(ops.l2norm(d["x"])), d["y"])


def test_gating():
    d = load("gating")
    HV = d["A_log"].shape[0]
    g, beta = ops.gdn_gating(d["A_log"], d["ba"][:, HV:], d["ba"][:, :HV], d["dt_bias"], ops.bf16)
    torch.testing.assert_close(g, d["g"], rtol=2e-5, atol=1e-6)
    assert torch.equal(beta, d["beta"])


def test_gdn_decode_step():
    d = load("gdn_decode")
    H, HV = d["H"], d["A_log"].shape[0]
    K = d["state_in"].shape[-1]
    mixed = d["mixed"].float()
    st = d["state_in"].clone()
    g, beta = ops.gdn_gating(d["A_log"], d["a"], d["b"], d["dt_bias"], ops.bf16)
    for i, s in enumerate(d["slots"].tolist()):
        if s < 0:
            assert bool((d["o"][i] == 0).all())
            continue
        q = ops.l2norm(mixed[i, :H * K].view(H, K))
        k = ops.l2norm(mixed[i, H * K:2 * H * K].view(H, K))
        v = mixed[i, 2 * H * K:].view(HV, K)
        o, st[s] = ops.gdn_recurrence(q[None], k[None], v[None], g[i:i + 1], beta[i:i + 1], st[s], K ** -0.5, HV // H)
        assert_bf16_close(ops.bf16(o[0]), d["o"][i, 0])
    torch.testing.assert_close(st, d["state_out"], rtol=2e-5, atol=2e-6)


def test_gated_norm():
    d = load("gated_norm")
    y = ops.gated_rmsnorm(d["x"], d["weight"], d["z"].reshape(-1, d["x"].shape[1]), 1e-6, ops.bf16)
    assert_bf16_close(y, d["y"])


def test_sigmoid_mul():
    d = load("sigmoid_mul")
    y = ops.sigmoid_mul(d["attn"], d["gate"].reshape(d["attn"].shape), ops.bf16)
    assert_bf16_close(y, d["y"])
