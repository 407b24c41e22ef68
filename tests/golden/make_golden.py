"""Generate golden input/output vectors from the reference's own Triton kernels.

Runs reference/qwen38_inference.py's kernels under the Triton CPU interpreter
(``TRITON_INTERPRET=1``) on small seeded inputs and writes ``tests/golden/*.pt``. This
needs a checkout of the reference (``--reference``); the fixtures it writes are committed
and the tests read only the fixtures.

Two fixes are applied to the stock interpreter so that it follows GPU semantics:
  * it stores bfloat16 as raw uint16 and applies numpy arithmetic to the bit patterns,
    so ``bf16 * bf16`` (used by the conv kernels, REF:384 and REF:1052) multiplied
    integers; bf16 binary ops are evaluated in fp32 and rounded to nearest-even instead;
  * its fp32 -> bf16 conversion truncated; it now rounds to nearest-even like
    ``cvt.rn.bf16.f32``.
Transcendentals then run as numpy fp32 (correctly rounded-ish), not as the GPU's
approximate instructions, so the oracle is compared against these vectors with a tolerance
of one bf16 ulp on rare elements (see tests/test_oracle_golden.py).

The reference's wrappers refuse CPU tensors in three places (eligibility check of the
decode conv, PDL capability probe, SM-count query); those host checks are bypassed, the
kernels and their launch code are the reference's.

Usage: python tests/golden/make_golden.py --reference <reference checkout>
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))


def _patch_interpreter():
    import triton.language as tl
    from triton.runtime import interpreter as I

    def f32_to_bf16_bits(a):
        return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)

    def bf16_bits_to_f32(a):
        return (np.ascontiguousarray(a).astype(np.uint32) << 16).view(np.float32)

    orig_cast = I.InterpreterBuilder.cast_impl
    orig_fp2fp = I.InterpreterBuilder.create_fp_to_fp
    orig_bin = I.InterpreterBuilder.binary_op

    def cast_impl(self, src, dst_type):
        s, d = src.dtype.scalar, dst_type.scalar
        if s == tl.float32 and d == tl.bfloat16:
            return I.TensorHandle(f32_to_bf16_bits(src.data), d)
        if s == tl.bfloat16 and d == tl.float32:
            return I.TensorHandle(bf16_bits_to_f32(src.data), d)
        return orig_cast(self, src, dst_type)

    def fp_to_fp(self, src, dst_type, rounding_mode):
        s, d = src.dtype.scalar, dst_type.scalar
        if (s, d) in ((tl.float32, tl.bfloat16), (tl.bfloat16, tl.float32)):
            return cast_impl(self, src, dst_type)
        return orig_fp2fp(self, src, dst_type, rounding_mode)

    def binary_op(self, lhs, rhs, op):
        if lhs.dtype.scalar == tl.bfloat16 and rhs.dtype.scalar == tl.bfloat16:
            out = op(bf16_bits_to_f32(lhs.data), bf16_bits_to_f32(rhs.data)).astype(np.float32)
            return I.TensorHandle(f32_to_bf16_bits(out), tl.bfloat16)
        return orig_bin(self, lhs, rhs, op)

    I.InterpreterBuilder.cast_impl = cast_impl
    I.InterpreterBuilder.create_fp_to_fp = fp_to_fp
    I.InterpreterBuilder.binary_op = binary_op
    for name in ("create_fadd", "create_fmul", "create_fdiv", "create_fsub", "create_precise_divf"):
        npop = {"create_fadd": np.add, "create_fmul": np.multiply, "create_fdiv": np.divide,
                "create_fsub": np.subtract, "create_precise_divf": np.divide}[name]
        setattr(I.InterpreterBuilder, name, (lambda op: (lambda self, a, b: binary_op(self, a, b, op)))(npop))
    for name in ("create_si_to_fp", "create_ui_to_fp", "create_fp_to_si", "create_fp_to_ui",
                 "create_fp_ext", "create_fp_trunc"):
        setattr(I.InterpreterBuilder, name, lambda self, src, dst_type: cast_impl(self, src, dst_type))


def _load_reference(root):
    sys.path.insert(0, str(root))
    import reference.qwen38_inference as R
    R.can_use_fused_qkvzba_causal_conv1d_update_contiguous = lambda *a, **k: (True, "cpu golden run")
    R.is_arch_support_pdl = lambda: False
    R._get_sm_count = lambda device: 148
    R._ENABLE_PDL = False
    # ``exp = tl.exp`` is a module-level alias (REF:74); the interpreter patches ``tl`` only
    # while a kernel runs, so resolve the alias at call time.
    import triton.language as tl
    R.exp = lambda x: tl.exp(x)

    class _NoDevice:
        def __init__(self, *_):
            pass

        def __enter__(self):
            return self

        def __exit__(self, *exc):
            return False

    R.device_context = _NoDevice
    return R


def bf(t):
    return t.to(torch.bfloat16)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="directory of the reference checkout")
    args = ap.parse_args()
    _patch_interpreter()
    R = _load_reference(Path(args.reference))
    from qwen38_inference_b200.config import HybridConfig, rope_table
    g = torch.Generator().manual_seed(1234)

    def rn(*shape, scale=1.0):
        return torch.randn(*shape, generator=g) * scale

    out = {}

    # K1: fused QK Gemma-RMSNorm + partial NeoX RoPE + gate split (REF:83-278)
    for tag, (nq, nkv, d, rd, T) in {"27b": (6, 1, 256, 64, 6), "tiny": (4, 2, 64, 16, 5)}.items():
        cfg = HybridConfig(hidden_size=64, intermediate_size=64, num_attention_heads=nq,
                           num_key_value_heads=nkv, head_dim=d, linear_num_key_heads=1,
                           linear_num_value_heads=1, linear_key_head_dim=64, linear_value_head_dim=64,
                           linear_conv_kernel_dim=4, num_hidden_layers=4, vocab_size=8,
                           partial_rotary_factor=rd / d)
        qkv = bf(rn(T, 2 * nq * d + 2 * nkv * d, scale=0.5))
        qg, k, _ = qkv.split([2 * nq * d, nkv * d, nkv * d], dim=-1)
        qw, kw = bf(rn(d, scale=0.1)), bf(rn(d, scale=0.1))
        rope = rope_table(cfg, 4096, "cpu")
        pos = torch.randint(0, 4096, (T,), generator=g)
        q_o, k_o, gate_o = R.fused_qk_gemma_rmsnorm_rope_gate(qg, k, qw, kw, rope, pos, 1e-6, nq, nkv, d, rd, has_gate=True)
        out[f"rope_{tag}"] = dict(qkv=qkv, q_w=qw, k_w=kw, rope=rope, positions=pos, nq=nq, nkv=nkv, d=d, rd=rd,
                                  q=q_o, k=k_o, gate=gate_o)

    # K2: decode conv update + z/b/a copies (REF:301-600); slot -1 is padding
    B, qk, vd, hv = 3, 128, 256, 2
    C = 2 * qk + vd
    qkvz = bf(rn(B, C + vd))
    ba = bf(rn(B, 2 * hv))
    st = bf(rn(4, C, 3))
    w = bf(rn(C, 4, scale=0.5))
    idx = torch.tensor([2, -1, 0], dtype=torch.int32)
    st_in = st.clone()
    mixed, z, b, a = R.fused_qkvzba_causal_conv1d_update_contiguous(
        qkvz, ba, st, w, None, idx, qkv_dim=C, v_dim=vd, num_v_heads=hv, head_v_dim=128, activation="silu")
    out["conv_decode"] = dict(qkvz=qkvz, ba=ba, state_in=st_in, weight=w, slots=idx, C=C,
                              mixed=mixed, z=z, b=b, a=a, state_out=st)

    # K4 + K3: prefill varlen conv with conv-state update (REF:704-1253, 603-699)
    lens = [5, 2, 1, 9, 3, 12]
    has = [True, True, False, False, True, False]
    slots = [3, 0, 1, 4, 2, 5]
    T = sum(lens)
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32)
    x_full = bf(rn(T, C + vd))  # qkvz-like buffer; conv reads the first C columns
    st = bf(rn(6, C, 3))
    st_in = st.clone()
    y = R.causal_conv1d_fn(x_full[:, :C].T, w, None, st, cu, lens, cache_indices=torch.tensor(slots, dtype=torch.int32),
                           has_initial_state=torch.tensor(has), activation="silu").T
    q_s, k_s, v_s = R.fused_qkv_split_gdn_prefill(y, 1, 1, 2, 128, 128, 128)
    out["conv_prefill"] = dict(x=x_full, weight=w, state_in=st_in, cu=cu, lens=lens, has_initial=has,
                               slots=slots, C=C, out=y.contiguous(), q=q_s[0], k=k_s[0], v=v_s[0], state_out=st)

    # K7: prefill l2 norm, bf16 out (REF:1550-1638 through REF:1738-1766)
    xq = bf(rn(9, 3, 128))
    out["l2norm"] = dict(x=xq, y=R.l2norm_fwd(xq, 1e-6))

    # K5: gating (REF:1258-1323)
    T5, HV = 7, 48
    ba5 = bf(rn(T5, 2 * HV))
    A_log = rn(HV)
    dt = bf(rn(HV))
    g5, beta5 = R.fused_gdn_gating(A_log, ba5[:, HV:], ba5[:, :HV], dt)
    out["gating"] = dict(ba=ba5, A_log=A_log, dt_bias=dt, g=g5[0], beta=beta5[0])

    # K6: decode recurrent step, in place, slot -1 writes zeros (REF:1328-1545)
    Bd, H, HVd, K = 3, 2, 6, 128
    mixed_d = bf(rn(Bd, 2 * H * K + HVd * K))
    a_d, b_d = bf(rn(Bd, HVd)), bf(rn(Bd, HVd))
    A_d, dt_d = rn(HVd), bf(rn(HVd))
    state = rn(3, HVd, K, K, scale=0.1)
    state_in = state.clone()
    o_d = torch.empty(Bd, 1, HVd, K, dtype=torch.bfloat16)
    idx_d = torch.tensor([1, -1, 2], dtype=torch.int32)
    R.fused_recurrent_gated_delta_rule_packed_decode(mixed_qkv=mixed_d, a=a_d, b=b_d, A_log=A_d, dt_bias=dt_d,
                                                     scale=K ** -0.5, initial_state=state, out=o_d,
                                                     ssm_state_indices=idx_d, use_qk_l2norm_in_kernel=True)
    out["gdn_decode"] = dict(mixed=mixed_d, a=a_d, b=b_d, A_log=A_d, dt_bias=dt_d, state_in=state_in, slots=idx_d,
                             H=H, o=o_d, state_out=state)

    # K9: gated RMSNorm, z as the strided 3-D view of the qkvz buffer (REF:1804-2089)
    Tn, HVn, dv = 5, 4, 128
    o_n = bf(rn(Tn * HVn, dv))
    zbuf = bf(rn(Tn, 3 * HVn * dv))
    zview = zbuf[:, HVn * dv:2 * HVn * dv].view(Tn, HVn, dv)
    wn = bf(rn(dv, scale=0.5) + 1.0)
    yn = R.rms_norm_gated(x=o_n, weight=wn, bias=None, z=zview, eps=1e-6, norm_before_gate=True, is_rms_norm=True,
                          activation="swish")
    out["gated_norm"] = dict(x=o_n, z=zview.contiguous(), weight=wn, y=yn)

    # K10: sigmoid gate multiply with the strided 3-D gate view (REF:2094-2175)
    Ts, nh, hd = 3, 6, 256
    att = bf(rn(Ts, nh * hd))
    gbuf = bf(rn(Ts, nh, 2 * hd))
    gview = gbuf[:, :, hd:]
    ys = R.fused_sigmoid_mul(att.clone(), gview, inplace=False)
    out["sigmoid_mul"] = dict(attn=att, gate=gview.contiguous(), y=ys)

    for name, d in out.items():
        torch.save(d, HERE / f"{name}.pt")
        print("wrote", name, {k: tuple(v.shape) for k, v in d.items() if isinstance(v, torch.Tensor)})


if __name__ == "__main__":
    main()
