"""Parity of the layer loop against the CPU oracle, unit by unit and at the model level.

Teacher forcing (``test_units_teacher_forced``): every half-layer unit of the GPU layer loop
(a mixer: attention or Gated DeltaNet with its output projection and the post-mixer
add-norm; or an MLP: gate_up with SwiGLU, down and the next layer's input add-norm) is fed
the oracle's state at that point, the normalized hidden rows and the residual, with the
layer's cache set to the oracle's cache before the call. Its output is compared with the
oracle's state after the same unit, in bf16 ulps, so a kernel error cannot hide behind the
rounding flips that a whole forward propagates. Two oracles are used for the GDN prefill
units: one with the kernel's chunked form and bf16 operands (oracle/chunked.py), which
bounds the kernels; and the reference's per-token recurrence, whose gap is recorded.

Model level (``test_logits_27b_width``): a 27B-width model (hidden 5120, MLP 17408, the
27B head counts) with 4 layers (3 GDN + 1 attention) and the full 248,320-entry vocabulary
runs prompts of 7 and 3 tokens and 4 decode steps (BASELINE configs[0]'s call pattern)
against the oracle. The reference harness's bound is atol = rtol = 1e-3
(test_forward_step.py:122-134), below one bf16 ulp of any |logit| > 0.25 since the logits
are float(bf16(h W^T)) (REF:5096): a single rounding flip anywhere upstream fails it. The
test asserts a floor on the fraction of logits within that bound and a bound on |d| in
logit ulps, and records both (printed; written to $QW_PARITY_OUT when set).

Units' bounds (bf16 ulps of the larger of the two values, with values below 2^-8 of their
row's largest magnitude counted at that floor): see UNIT_ULPS.
"""
import json
import os

import pytest
import torch

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16

# unit kind -> largest difference allowed, bf16 ulps, for hidden (normalized) and residual
UNIT_ULPS = {"mlp": (4.0, 2.0), "attn": (4.0, 2.0), "gdn_decode": (4.0, 2.0), "gdn_prefill": (4.0, 2.0)}
# GDN prefill against the per-token recurrence (the reference's definition), recorded and
# bounded loosely: the chunked form's bf16 operands move o by up to ~1e-2 of its scale
GDN_TOKEN_ULPS = (64.0, 16.0)
# model level: fraction of logits within atol = rtol = 1e-3, and the largest |d| in bf16 ulps
LOGIT_FRAC_FLOOR = 0.5
LOGIT_MAX_ULPS = 8.0


def ulps(got, exp):
    got, exp = got.float().cpu(), exp.float().cpu()
    row = torch.maximum(got.abs(), exp.abs()).amax(dim=-1, keepdim=True)
    mag = torch.maximum(torch.maximum(got.abs(), exp.abs()), row * 2.0 ** -8).clamp_min(2.0 ** -126)
    return (got - exp).abs() / torch.exp2(torch.floor(torch.log2(mag)) - 7)


def _record(key, value):
    path = os.environ.get("QW_PARITY_OUT")
    if not path:
        return
    data = {}
    if os.path.exists(path):
        with open(path) as f:
            data = json.load(f)
    data[key] = value
    with open(path, "w") as f:
        json.dump(data, f, indent=1)


@pytest.fixture(scope="module")
def wide():
    """27B width, 4 layers, full vocabulary; weights drawn on the GPU, the oracle's copy on
    the host."""
    from oracle import OracleModel
    from qwen38_inference_b200 import Qwen38
    from qwen38_inference_b200.config import HybridConfig, qwen38_27b, random_weights
    import dataclasses
    cfg = dataclasses.replace(qwen38_27b(), num_hidden_layers=4)
    assert isinstance(cfg, HybridConfig) and cfg.layer_types[3] == "full_attention"
    w = random_weights(cfg, seed=7, device="cuda")
    gpu = Qwen38(config=cfg, weights=w, device="cuda:0", max_context=512)
    wc = {k: v.cpu() for k, v in w.items()}
    del w
    torch.cuda.empty_cache()
    ref = OracleModel(cfg, wc, dtype=BF16, max_context=512)
    ref_ch = OracleModel(cfg, wc, dtype=BF16, max_context=512, gdn_prefill_form="chunked")
    return cfg, gpu, ref, ref_ch


def _load_layer(gc, rc, i):
    if i in rc.kv:
        gc.kv[i][0].copy_(rc.kv[i][0])
        gc.kv[i][1].copy_(rc.kv[i][1])
    else:
        gc.conv[i].copy_(rc.conv[i])
        gc.recurrent[i].copy_(rc.recurrent[i])


def _calls(vocab):
    g = torch.Generator().manual_seed(12)
    ids = lambda n: torch.randint(vocab, (n,), generator=g).tolist()  # noqa: E731
    # configs[0]'s pattern, then a ragged prefill over several chunks on top of the cached
    # prefixes (cached-prefix attention and a carried GDN state), then one more decode
    return [([ids(7), ids(3)], [0, 1]), ([ids(1), ids(1)], [0, 1]), ([ids(1), ids(1)], [0, 1]),
            ([ids(130), ids(70)], [1, 0]), ([ids(1), ids(1)], [0, 1])]


@torch.inference_mode()
def test_units_teacher_forced(wide):
    cfg, gpu, ref, ref_ch = wide
    B, cap = 2, 256  # no growth: both caches keep one layout
    n_units = 2 * cfg.num_hidden_layers
    rc, rcc = ref.new_cache(B, initial_capacity=cap), ref_ch.new_cache(B, initial_capacity=cap)
    gc = gpu.new_cache(B, initial_capacity=cap)
    stats = {}
    for call, (rows, slots) in enumerate(_calls(cfg.vocab_size)):
        lens = [len(r) for r in rows]
        prefixes = [rc.lengths[s] for s in slots]
        is_decode = all(n == 1 and p > 0 for n, p in zip(lens, prefixes))
        flat = [t for r in rows for t in r]
        before, before_ch = rc.clone(), rcc.clone()
        tr, tr_ch = [], []
        ref.forward_step(rows, rc, request_indices=slots, trace=tr)
        ref_ch.forward_step(rows, rcc, request_indices=slots, trace=tr_ch)
        assert len(tr) == n_units + 1
        for u in range(n_units):
            i = u // 2
            kind = "mlp" if u % 2 else ("attn" if cfg.layer_types[i] == "full_attention" else
                                        ("gdn_decode" if is_decode else "gdn_prefill"))
            forms = [("chunked", tr_ch, before_ch, rcc)] if kind == "gdn_prefill" else []
            forms.append(("token", tr, before, rc))
            for form, trace, pre, post in forms:
                _load_layer(gc, pre, i)
                h = trace[u][0].to(BF16).cuda()
                r = trace[u][1].to(BF16).cuda()
                gpu._engine.run_units(flat, slots, prefixes, lens, gc, is_decode, (u, u + 1), h, r)
                torch.cuda.synchronize()
                uh, ur = ulps(h, trace[u + 1][0]), ulps(r, trace[u + 1][1])
                key = kind if form == "chunked" or kind != "gdn_prefill" else "gdn_prefill_vs_token"
                st = stats.setdefault(key, {"hidden_max_ulps": 0.0, "resid_max_ulps": 0.0, "n": 0,
                                            "hidden_frac_over_1ulp": 0.0, "resid_frac_over_1ulp": 0.0})
                st["hidden_max_ulps"] = max(st["hidden_max_ulps"], uh.max().item())
                st["resid_max_ulps"] = max(st["resid_max_ulps"], ur.max().item())
                st["hidden_frac_over_1ulp"] = max(st["hidden_frac_over_1ulp"], (uh > 1).float().mean().item())
                st["resid_frac_over_1ulp"] = max(st["resid_frac_over_1ulp"], (ur > 1).float().mean().item())
                st["n"] += 1
                if u % 2 == 0 and form != "token" or (u % 2 == 0 and kind != "gdn_prefill"):
                    # the mixer's cache writes: KV rows of this call, conv state, recurrent state
                    if i in post.kv:
                        loc = [64 + s * cap + p + j for s, p, n in zip(slots, prefixes, lens) for j in range(n)]
                        for a, b in zip(gc.kv[i], post.kv[i]):
                            ku = ulps(a[loc].cpu().flatten(1), b[loc].flatten(1))
                            st["kv_max_ulps"] = max(st.get("kv_max_ulps", 0.0), ku.max().item())
                    else:
                        cu_ = ulps(gc.conv[i].cpu().flatten(1), post.conv[i].flatten(1))
                        st["conv_max_ulps"] = max(st.get("conv_max_ulps", 0.0), cu_.max().item())
                        sg, se = gc.recurrent[i].cpu(), post.recurrent[i]
                        rel = ((sg - se).abs().max() / se.abs().max().clamp_min(1e-30)).item()
                        st["state_rel"] = max(st.get("state_rel", 0.0), rel)
    print("teacher-forced units:", json.dumps(stats, indent=1))
    _record("units_27b_width", stats)
    for kind, (bh, br) in UNIT_ULPS.items():
        st = stats[kind]
        assert st["hidden_max_ulps"] <= bh and st["resid_max_ulps"] <= br, (kind, st)
        assert st.get("kv_max_ulps", 0.0) <= 2.0 and st.get("conv_max_ulps", 0.0) <= 2.0, (kind, st)
        assert st.get("state_rel", 0.0) <= 1e-3, (kind, st)
    st = stats["gdn_prefill_vs_token"]
    assert st["hidden_max_ulps"] <= GDN_TOKEN_ULPS[0] and st["resid_max_ulps"] <= GDN_TOKEN_ULPS[1], st


def test_logits_27b_width(wide):
    cfg, gpu, ref, _ = wide
    g = torch.Generator().manual_seed(0)
    ids = lambda n: torch.randint(cfg.vocab_size, (n,), generator=g).tolist()  # noqa: E731
    steps = [[ids(7), ids(3)]] + [[ids(1), ids(1)] for _ in range(4)]
    rc, gc = ref.new_cache(2, initial_capacity=64), gpu.new_cache(2, initial_capacity=64)
    recs = []
    for rows in steps:
        exp = ref.forward_step([list(r) for r in rows], rc)
        got = gpu.forward_step([list(r) for r in rows], gc).cpu()
        assert got.shape == exp.shape and bool(torch.isfinite(got).all())
        assert gc.lengths == rc.lengths and gc.capacity == rc.capacity
        d = (got - exp).abs()
        within = (d <= 1e-3 + 1e-3 * exp.abs()).float().mean().item()
        # logits are float(bf16(.)): their differences come in whole bf16 ulps
        lu = ulps(got, exp)
        top_same = (got.argmax(-1) == exp.argmax(-1)).float().mean().item()
        recs.append({"frac_within_1e-3": round(within, 5), "max_abs_diff": d.max().item(),
                     "max_ulps": lu.max().item(), "frac_over_1ulp": (lu > 1).float().mean().item(),
                     "argmax_agree": top_same})
    print("27B-width logits per call:", json.dumps(recs, indent=1))
    _record("logits_27b_width", recs)
    gpu.check_device_error()
    for r in recs:
        assert r["frac_within_1e-3"] >= LOGIT_FRAC_FLOOR, recs
        assert r["max_ulps"] <= LOGIT_MAX_ULPS, recs
