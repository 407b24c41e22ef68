"""The kernel-rounding restatement of the chunked delta rule (oracle/chunked.py) against the
per-token fp32 recurrence (oracle/ops.py gdn_recurrence, REF:1355-1408).

* With its operand rounding switched off, the restatement is the chunk algebra alone and
  agrees with the recurrence to fp32 accuracy (1e-5 of each head's output scale).
* With the kernel's bf16 / tf32 operand rounding (the form of the reference's flashinfer
  chunked kernel, REF:5084), the outputs move by at most 2e-2 of each head's largest
  |o| and the final state by at most 1e-2 of its largest entry: the size of the gap that
  the prefill kernel's GPU test attributes to the algorithm rather than to the kernel.
"""
import pytest
import torch

from oracle import ops as O
from oracle.chunked import chunked_gdn, tf32


def bf(t):
    return t.bfloat16().float()


def test_tf32_rounding():
    x = torch.tensor([1.0, 1 + 2 ** -11, 1 + 3 * 2 ** -11, -1 - 2 ** -11, 1 + 2 ** -12, 3.0])
    assert tf32(x).tolist() == [1.0, 1 + 2 ** -10, 1 + 2 * 2 ** -10, -1 - 2 ** -10, 1.0, 3.0]


def _case(n, seed, HV=6, H=2, dk=128):
    g = torch.Generator().manual_seed(seed)
    q = bf(O.l2norm(torch.randn(n, H, dk, generator=g)))
    k = bf(O.l2norm(torch.randn(n, H, dk, generator=g)))
    v = bf(torch.randn(n, HV, dk, generator=g))
    ba = bf(torch.randn(n, 2 * HV, generator=g))
    A_log = torch.randn(HV, generator=g) * 0.5
    dt = bf(torch.randn(HV, generator=g) * 0.5)
    state = torch.randn(HV, dk, dk, generator=g) * 0.05
    return q, k, v, ba, A_log, dt, state


@pytest.mark.parametrize("n", [1, 64, 65, 200])
def test_chunked_restatement_against_token_recurrence(n):
    HV, H, dk = 6, 2, 128
    q, k, v, ba, A_log, dt, state = _case(n, 40 + n, HV, H, dk)
    a, b = ba[:, HV:], ba[:, :HV]
    gg, beta = O.gdn_gating(A_log, a, b, dt, O.bf16)
    o_ref, s_ref = O.gdn_recurrence(q, k, v, gg, beta, state, dk ** -0.5, HV // H)
    scale = o_ref.abs().amax(dim=(0, 2), keepdim=True)
    o, s = chunked_gdn(q, k, v, a, b, A_log, dt, state, dk ** -0.5, HV // H, operand_rounding=False)
    assert ((o - o_ref).abs() / scale).max() < 1e-5
    assert (s - s_ref).abs().max() / s_ref.abs().max() < 1e-5
    o, s = chunked_gdn(q, k, v, a, b, A_log, dt, state, dk ** -0.5, HV // H)
    assert torch.equal(o, bf(o))  # o is rounded to bf16, as the kernel stores it
    err_o = ((o - o_ref).abs() / scale).max().item()
    err_s = ((s - s_ref).abs().max() / s_ref.abs().max()).item()
    assert err_o < 2e-2 and err_s < 1e-2, (err_o, err_s)
