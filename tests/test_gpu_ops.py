"""Per-kernel parity: every sm_100a op against the CPU oracle op (oracle/ops.py) on the same
seeded inputs, with the 27B per-head geometry.

Tolerances (bf16 outputs): an element may differ from the oracle by a few bf16 ulps of its
magnitude plus a small absolute term; the fraction of differing elements is bounded. The
oracle computes in fp32 with the reference's rounding points; the kernels reach the same
rounding points with a different fp32 summation order, so isolated last-ulp flips are
expected. Cache bookkeeping (rows written, state shifts, growth copies) is bit-exact.
"""
import pytest
import torch

from oracle import ops as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def K():
    from qwen38_inference_b200 import ops
    return ops


def bf(t):
    return t.to(torch.bfloat16)


def ulp(x):
    x = x.float().abs().clamp_min(2.0 ** -126)
    return torch.exp2(torch.floor(torch.log2(x)) - 7)


def close(got, exp, n_ulp=2.0, atol=1e-5, max_frac=0.05):
    got, exp = got.float().cpu(), exp.float().cpu()
    d = (got - exp).abs()
    bound = n_ulp * torch.maximum(ulp(got), ulp(exp)) + atol
    bad = d > bound
    assert not bool(bad.any()), f"{int(bad.sum())}/{d.numel()} beyond bound; max diff {d.max().item():.3g}"
    frac = (d > 0).float().mean().item()
    assert frac <= max_frac, f"{frac:.3f} of elements differ"


def close_rows(got, exp, n_ulp, max_frac):
    """Like close(), in bf16 ulps of max(|element|, RMS of its row along the last dimension):
    an element that cancellation made small (a rotated pair) is measured at its row's scale."""
    got, exp = got.float().cpu(), exp.float().cpu()
    d = (got - exp).abs()
    rms = exp.pow(2).mean(dim=-1, keepdim=True).sqrt()
    u = d / ulp(torch.maximum(torch.maximum(got.abs(), exp.abs()), rms))
    assert not bool((u > n_ulp).any()), f"{int((u > n_ulp).sum())}/{d.numel()} beyond {n_ulp} ulps; max {u.max().item():.2f}"
    assert (d > 0).float().mean().item() <= max_frac


def gen(seed):
    return torch.Generator().manual_seed(seed)


def test_embed_and_add_rmsnorm(K):
    g = gen(1)
    V, H, T = 500, 5120, 37
    table = bf(torch.randn(V, H, generator=g))
    w = bf(torch.randn(H, generator=g) * 0.1)
    tok = torch.randint(V, (T,), generator=g, dtype=torch.int32)
    resid = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
    hid = torch.empty_like(resid)
    K.embed_rmsnorm(tok.to(DEV), table.to(DEV), w.to(DEV), resid, hid, 1e-6)
    assert torch.equal(resid.cpu(), table[tok.long()])
    close(hid, O.gemma_rmsnorm(table[tok.long()], w, 1e-6, O.bf16), n_ulp=1)
    x = bf(torch.randn(T, H, generator=g))
    r = bf(torch.randn(T, H, generator=g))
    xd, rd = x.to(DEV), r.to(DEV)
    K.add_rmsnorm(xd, rd, w.to(DEV), 1e-6)
    ex, er = O.gemma_add_rmsnorm(x, r, w, 1e-6, O.bf16)
    assert torch.equal(rd.cpu().float(), er)  # residual = bf16(x + r) exactly
    close(xd, ex, n_ulp=1)
    rows = torch.tensor([3, 0, 36], dtype=torch.int32)
    out = torch.empty(3, H, dtype=torch.bfloat16, device=DEV)
    K.add_rmsnorm_rows(x.to(DEV), r.to(DEV), w.to(DEV), out, 1e-6, rows.to(DEV))
    close(out, ex[rows.long()], n_ulp=1)


def test_gated_rmsnorm(K):
    g = gen(2)
    T, HV, D = 19, 48, 128
    x = bf(torch.randn(T, HV * D, generator=g))
    zbuf = bf(torch.randn(T, 3 * HV * D, generator=g))
    z = zbuf[:, HV * D:2 * HV * D]
    w = bf(torch.randn(D, generator=g) * 0.3 + 1)
    y = torch.empty(T, HV * D, dtype=torch.bfloat16, device=DEV)
    zd = zbuf.to(DEV)[:, HV * D:2 * HV * D]
    K.gated_rmsnorm(x.to(DEV), zd, w.to(DEV), y, HV, D, 1e-6)
    exp = O.gated_rmsnorm(x.reshape(-1, D), w, z.reshape(-1, D), 1e-6, O.bf16).reshape(T, -1)
    close(y, exp, n_ulp=2)


@pytest.mark.parametrize("nq,nkv,d,rd", [(24, 4, 256, 64), (6, 1, 256, 64), (4, 2, 64, 16)])
def test_qk_norm_rope_store(K, nq, nkv, d, rd):
    from qwen38_inference_b200.config import rope_table, HybridConfig
    g = gen(3)
    T, rows = 11, 200
    cfg = HybridConfig(hidden_size=64, intermediate_size=64, num_attention_heads=nq, num_key_value_heads=nkv,
                       head_dim=d, linear_num_key_heads=1, linear_num_value_heads=1, linear_key_head_dim=128,
                       linear_value_head_dim=128, linear_conv_kernel_dim=4, num_hidden_layers=4, vocab_size=8,
                       partial_rotary_factor=rd / d)
    rope = rope_table(cfg, 1024, DEV)
    qkv = bf(torch.randn(T, 2 * nq * d + 2 * nkv * d, generator=g))
    qw, kw = bf(torch.randn(d, generator=g) * 0.1), bf(torch.randn(d, generator=g) * 0.1)
    pos = torch.randint(0, 1024, (T,), generator=g, dtype=torch.int32)
    loc = torch.randperm(rows - 64, generator=g)[:T].to(torch.int32) + 64
    kc = torch.full((rows, nkv, d), float("nan"), dtype=torch.bfloat16, device=DEV)  # poisoned
    vc = torch.full_like(kc, float("nan"))
    qd = qkv.to(DEV)
    K.qk_norm_rope_store(qd, nq, nkv, d, qw.to(DEV), kw.to(DEV), rope, pos.to(DEV), loc.to(DEV), kc, vc, 1e-6)
    qg, k, v = qkv.float().split([2 * nq * d, nkv * d, nkv * d], dim=-1)
    eq, ek, _ = O.qk_norm_rope_gate(qg, k, qw, kw, rope.cpu(), pos.long(), 1e-6, nq, nkv, d, rd, O.bf16)
    got_q = qd.cpu().float()[:, :2 * nq * d].view(T, nq, 2 * d)
    close(got_q[..., :d], eq, n_ulp=1)
    assert torch.equal(got_q[..., d:], qg.view(T, nq, 2 * d)[..., d:])  # gate untouched
    close(kc.cpu()[loc.long()], ek, n_ulp=1)
    assert torch.equal(vc.cpu()[loc.long()].float(), v.view(T, nkv, d))
    untouched = torch.ones(rows, dtype=torch.bool)
    untouched[loc.long()] = False
    assert bool(torch.isnan(kc.cpu()[untouched].float()).all())


def _attn_case(g, nq, nkv, d, prefixes, lens, cap=512):
    S = len(lens)
    rows = S * cap + 64
    kc = bf(torch.randn(rows, nkv, d, generator=g))
    vc = bf(torch.randn(rows, nkv, d, generator=g))
    T = sum(lens)
    qkv = bf(torch.randn(T, 2 * nq * d + 2 * nkv * d, generator=g))
    starts = [64 + s * cap for s in range(S)]
    return kc, vc, qkv, starts


@pytest.mark.parametrize("nq,nkv,d,case", [(24, 4, 256, "mixed"), (6, 1, 256, "mixed"), (4, 2, 64, "mixed"),
                                           (24, 4, 256, "long"), (4, 2, 64, "long")])
def test_attn_prefill(K, nq, nkv, d, case):
    """Causal varlen attention: ragged requests with cached prefixes; "long" has several
    query tiles and key blocks with growing score magnitudes (the running max rises
    across blocks, so rows of O are rescaled in TMEM)."""
    from qwen38_inference_b200.model import build_metadata
    g = gen(4)
    if case == "mixed":
        prefixes, lens = [0, 37, 130, 0], [200, 1, 77, 129]
    else:
        prefixes, lens = [0, 300], [700, 260]
    kc, vc, qkv, starts = _attn_case(g, nq, nkv, d, prefixes, lens, cap=1024)
    if case == "long":
        # keys grow in magnitude with their position: later blocks raise the row max
        pos = torch.arange(kc.shape[0], dtype=torch.float32).view(-1, 1, 1)
        kc = bf(kc.float() * (1.0 + pos / 256.0))
    packed, offs, T = build_metadata(list(range(len(lens))), prefixes, lens, 1024)
    md = {k: torch.from_numpy(packed[o:o + n]).to(DEV) for k, (o, n) in offs.items()}
    out = torch.empty(T, nq * d, dtype=torch.bfloat16, device=DEV)
    K.attn_prefill(qkv.to(DEV), nq, nkv, d, kc.to(DEV), vc.to(DEV), md["tiles"], md["cu"], md["prefix"],
                   md["kv_base"], out, d ** -0.5)
    q = qkv.float()[:, :2 * nq * d].view(T, nq, 2 * d)
    att = O.paged_attention(q[..., :d], kc, vc, starts, prefixes, lens, d ** -0.5, O.bf16)
    exp = O.sigmoid_mul(att.reshape(T, -1), q[..., d:].reshape(T, -1), O.bf16)
    # P is rounded to bf16 before the PV product (tensor cores): allow a few ulps. With the
    # peaked rows of the "long" case (a few keys carry almost all the weight) that rounding
    # reaches ~2^-7 of |v| on isolated outputs.
    close(out, exp, n_ulp=4, atol=2e-3 if case == "mixed" else 1.6e-2, max_frac=0.5)


@pytest.mark.parametrize("nq,nkv,d", [(24, 4, 256), (3, 1, 256), (4, 2, 64)])
@pytest.mark.parametrize("splits", [4, 0])
def test_attn_prefill_split_kv(K, nq, nkv, d, splits):
    """Prefill attention with every tile's keys split over CTAs (long cached prefixes, as in
    chunked prefill of one long request; nq = 3, nkv = 1 is an 8-way tensor-parallel rank),
    against the oracle and against the unsplit kernel. splits = 0 takes the engine's choice.
    A split whose key range lies beyond a row's causal limit contributes nothing to it."""
    from qwen38_inference_b200.model import build_metadata
    g = gen(6)
    prefixes, lens = [3000, 0, 5000], [512, 130, 64]
    cap = 8192
    kc, vc, qkv, starts = _attn_case(g, nq, nkv, d, prefixes, lens, cap=cap)
    packed, offs, T = build_metadata(list(range(len(lens))), prefixes, lens, cap)
    md = {k: torch.from_numpy(packed[o:o + n]).to(DEV) for k, (o, n) in offs.items()}
    n_tiles = md["tiles"].numel() // 2
    if splits == 0:
        splits = K.prefill_attn_splits(nq, n_tiles, max(p + n for p, n in zip(prefixes, lens)))
        assert (splits > 1) == (nq * n_tiles < 148)  # 24 heads x 7 tiles already fill the SMs
    args = (qkv.to(DEV), nq, nkv, d, kc.to(DEV), vc.to(DEV), md["tiles"], md["cu"], md["prefix"], md["kv_base"])
    whole = torch.empty(T, nq * d, dtype=torch.bfloat16, device=DEV)
    K.attn_prefill(*args, whole, d ** -0.5)
    out = torch.full((T, nq * d), float("nan"), dtype=torch.bfloat16, device=DEV)
    K.attn_prefill(*args, out, d ** -0.5, splits=splits, ws=K.Workspace(DEV))
    q = qkv.float()[:, :2 * nq * d].view(T, nq, 2 * d)
    att = O.paged_attention(q[..., :d], kc, vc, starts, prefixes, lens, d ** -0.5, O.bf16)
    exp = O.sigmoid_mul(att.reshape(T, -1), q[..., d:].reshape(T, -1), O.bf16)
    close(out, exp, n_ulp=4, atol=2e-3, max_frac=0.5)
    # each split keeps its own lazily raised running max, so P is rounded to bf16 at other
    # scales than in the unsplit kernel: many outputs move by an ulp, none by more than two
    close(out, whole, n_ulp=2, atol=1e-3, max_frac=0.6)


@pytest.mark.parametrize("nq,nkv,d", [(24, 4, 256), (4, 2, 64)])
@pytest.mark.parametrize("splits", [1, 3])
def test_attn_decode(K, nq, nkv, d, splits):
    g = gen(5)
    lens = [1] * 5
    prefixes = [1, 63, 64, 300, 511]
    kc, vc, qkv, starts = _attn_case(g, nq, nkv, d, prefixes, lens)
    B = len(lens)
    seq_len = torch.tensor([p + 1 for p in prefixes], dtype=torch.int32)
    kv_base = torch.tensor(starts, dtype=torch.int32)
    out = torch.empty(B, nq * d, dtype=torch.bfloat16, device=DEV)
    ws = K.Workspace(DEV)
    K.attn_decode(qkv.to(DEV), B, nq, nkv, d, kc.to(DEV), vc.to(DEV), seq_len.to(DEV), kv_base.to(DEV), 512, splits,
                  out, d ** -0.5, ws)
    q = qkv.float()[:, :2 * nq * d].view(B, nq, 2 * d)
    att = O.paged_attention(q[..., :d], kc, vc, starts, prefixes, lens, d ** -0.5, O.bf16)
    exp = O.sigmoid_mul(att.reshape(B, -1), q[..., d:].reshape(B, -1), O.bf16)
    # P is rounded to bf16 before the PV product (tensor cores), as in prefill
    close(out, exp, n_ulp=4, atol=2e-3, max_frac=0.5)


def test_conv_prefill(K):
    g = gen(6)
    H, HV, dk = 2, 6, 128
    qk, vd = H * dk, HV * dk
    C = 2 * qk + vd
    lens, has, slots = [5, 2, 1, 70, 3, 130], [1, 1, 0, 1, 0, 1], [3, 0, 1, 4, 2, 5]
    T = sum(lens)
    x = bf(torch.randn(T, C + vd, generator=g))
    w = bf(torch.randn(C, 4, generator=g) * 0.5)
    st = bf(torch.randn(6, C, 3, generator=g))
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    std = st.to(DEV)
    qo = torch.empty(T, qk, dtype=torch.bfloat16, device=DEV)
    ko, vo = torch.empty_like(qo), torch.empty(T, vd, dtype=torch.bfloat16, device=DEV)
    t32 = lambda a: torch.tensor(a, dtype=torch.int32, device=DEV)
    K.conv_prefill(x.to(DEV), w.to(DEV), std, t32(cu), t32(slots), t32(has), len(lens), max(lens), qo, ko, vo, qk, vd,
                   dk)
    ex_st = st.clone()
    y = O.conv_prefill(x[:, :C], w, ex_st, cu, slots, [bool(h) for h in has], O.bf16)
    assert torch.equal(std.cpu(), ex_st)  # conv state = last 3 raw inputs, bit-exact
    close(vo, y[:, 2 * qk:], n_ulp=1, max_frac=0.02)
    eq = O.bf16(O.l2norm(y[:, :qk].reshape(T, H, dk))).reshape(T, qk)
    ek = O.bf16(O.l2norm(y[:, qk:2 * qk].reshape(T, H, dk))).reshape(T, qk)
    close(qo, eq, n_ulp=2, max_frac=0.05)
    close(ko, ek, n_ulp=2, max_frac=0.05)


# bf16 ulps allowed between the chunked prefill kernel and oracle/chunked.py
GDN_CHUNK_ULPS = 4.0


def _gdn_inputs(g, lens, H=2, HV=6, S=None):
    dk = 128
    T = sum(lens)
    S = S or len(lens)
    q = bf(O.l2norm(torch.randn(T, H, dk, generator=g)))
    k = bf(O.l2norm(torch.randn(T, H, dk, generator=g)))
    v = bf(torch.randn(T, HV, dk, generator=g))
    ba = bf(torch.randn(T, 2 * HV, generator=g))
    A_log = torch.randn(HV, generator=g) * 0.5
    dt = bf(torch.randn(HV, generator=g) * 0.5)
    state = torch.randn(S, HV, dk, dk, generator=g) * 0.05
    return q, k, v, ba, A_log, dt, state


@pytest.mark.parametrize("lens", [[64], [1, 63, 65, 130], [200, 7], [257], [0, 129, 3], [600, 1, 64, 448]])
def test_gdn_prefill_chunked(K, lens):
    g = gen(7)
    H, HV, dk = 2, 6, 128
    q, k, v, ba, A_log, dt, state = _gdn_inputs(g, lens, H, HV, S=len(lens) + 1)
    slots = list(range(len(lens)))[::-1]
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    T = cu[-1]
    zbuf = bf(torch.randn(T, 2 * HV * dk, generator=g))  # z is a strided view, as in the qkvz buffer
    norm_w = bf(torch.randn(dk, generator=g) * 0.3 + 1)
    sd = state.to(DEV)
    y = torch.empty(T, HV * dk, dtype=torch.bfloat16, device=DEV)
    t32 = lambda a: torch.tensor(a, dtype=torch.int32, device=DEV)
    zd = zbuf.to(DEV)[:, HV * dk:]
    K.gdn_prefill(q.to(DEV), k.to(DEV), v.to(DEV), ba.to(DEV), A_log.to(DEV), dt.to(DEV), t32(cu), t32(slots),
                  len(lens), sd, zd, norm_w.to(DEV), y, H, HV, dk, dk, dk ** -0.5, 1e-6)
    gg, beta = O.gdn_gating(A_log, ba[:, HV:], ba[:, :HV], dt, O.bf16)
    exp_state = state.clone()
    exp_o = torch.empty(T, HV, dk)
    for i, s in enumerate(slots):
        a0, a1 = cu[i], cu[i + 1]
        exp_o[a0:a1], exp_state[s] = O.gdn_recurrence(q[a0:a1], k[a0:a1], v[a0:a1], gg[a0:a1], beta[a0:a1],
                                                      state[s], dk ** -0.5, HV // H)
    exp_y = O.gated_rmsnorm(O.bf16(exp_o).reshape(-1, dk), norm_w, zbuf[:, HV * dk:].reshape(-1, dk), 1e-6,
                            O.bf16).reshape(T, HV, dk)
    got = y.cpu().float().view(T, HV, dk)
    got_state = sd.cpu()
    # 1) against the kernel-rounding restatement of the chunked form (oracle/chunked.py):
    # the same bf16 / tf32 operands, so what is left is fp32 summation order and the rare
    # bf16 rounding flip it causes in an operand tile; bounded in bf16 ulps (of an element, or
    # of its (token, head) row's RMS where it is smaller); the state to 1e-2 of its largest
    # entry (one flipped U element moves a row of S by ~2^-8 of that element's share)
    from oracle.chunked import chunked_gdn
    ch_state = state.clone()
    ch_o = torch.empty(T, HV, dk)
    for i, s in enumerate(slots):
        a0, a1 = cu[i], cu[i + 1]
        ch_o[a0:a1], ch_state[s] = chunked_gdn(q[a0:a1], k[a0:a1], v[a0:a1], ba[a0:a1, HV:], ba[a0:a1, :HV], A_log, dt,
                                               state[s], dk ** -0.5, HV // H)
    ch_y = O.gated_rmsnorm(ch_o.reshape(-1, dk), norm_w, zbuf[:, HV * dk:].reshape(-1, dk), 1e-6,
                           O.bf16).reshape(T, HV, dk)
    d = (got - ch_y).abs()
    rms = ch_y.pow(2).mean(dim=-1, keepdim=True).sqrt()
    # bf16 ulps of max(|element|, RMS of its (token, head) row)
    n_ulp = d / ulp(torch.maximum(torch.maximum(got.abs(), ch_y.abs()), rms))
    bad = n_ulp > GDN_CHUNK_ULPS
    assert not bool(bad.any()), f"{int(bad.sum())} outputs beyond {GDN_CHUNK_ULPS} ulps; max {n_ulp.max().item():.1f} ulps"
    serr_ch = ((got_state - ch_state).abs().max() / ch_state.abs().max()).item()
    assert serr_ch < 1e-2, f"state vs the chunked restatement: {serr_ch}"
    # 2) against the per-token fp32 recurrence (the reference's definition): the bf16
    # operands of the chunked form move the output by up to ~1e-2 of its scale (the size the
    # CPU test of oracle/chunked.py measures between the two oracles), hence 3e-2 here
    scale = exp_y.abs().amax(dim=-1, keepdim=True).clamp_min(1e-3)
    err = ((got - exp_y).abs() / scale).max().item()
    assert err < 3e-2, f"relative output error {err}"
    serr = ((got_state - exp_state).abs().max() / exp_state.abs().max()).item()
    assert serr < 2e-2, f"relative state error {serr}"
    untouched = [s for s in range(len(lens) + 1) if s not in slots]
    for s in untouched:
        assert torch.equal(got_state[s], state[s])
    print("gdn chunked: vs restatement max", round(n_ulp.max().item(), 2), "ulps,",
          f"{(d > 0).float().mean().item():.4f} of outputs differ, state {serr_ch:.2e};",
          "vs token recurrence: output", round(err, 5), "state", round(serr, 6))


def test_gdn_decode_fused(K):
    g = gen(8)
    H, HV, dk = 2, 6, 128
    B, S = 4, 6
    C = 2 * H * dk + HV * dk
    qkvz = bf(torch.randn(B, C + HV * dk, generator=g))
    ba = bf(torch.randn(B, 2 * HV, generator=g))
    conv_w = bf(torch.randn(C, 4, generator=g) * 0.5)
    conv_state = bf(torch.randn(S, C, 3, generator=g))
    state = torch.randn(S, HV, dk, dk, generator=g) * 0.05
    A_log, dt = torch.randn(HV, generator=g) * 0.5, bf(torch.randn(HV, generator=g) * 0.5)
    norm_w = bf(torch.randn(dk, generator=g) * 0.3 + 1)
    slots = [4, 0, 5, 2]
    csd, sd = conv_state.to(DEV), state.to(DEV)
    y = torch.empty(B, HV * dk, dtype=torch.bfloat16, device=DEV)
    K.gdn_decode(qkvz.to(DEV), ba.to(DEV), conv_w.to(DEV), csd, sd, torch.tensor(slots, dtype=torch.int32, device=DEV),
                 B, A_log.to(DEV), dt.to(DEV), norm_w.to(DEV), y, H, HV, dk, dk, 1e-6)
    ecs, est = conv_state.clone(), state.clone()
    mixed = O.conv_decode(qkvz[:, :C], conv_w, ecs, slots, O.bf16)
    assert torch.equal(csd.cpu(), ecs)
    gg, beta = O.gdn_gating(A_log, ba[:, HV:], ba[:, :HV], dt, O.bf16)
    qn = O.l2norm(mixed[:, :H * dk].reshape(B, H, dk))
    kn = O.l2norm(mixed[:, H * dk:2 * H * dk].reshape(B, H, dk))
    v = mixed[:, 2 * H * dk:].reshape(B, HV, dk)
    o = torch.empty(B, HV, dk)
    for i, s in enumerate(slots):
        oo, est[s] = O.gdn_recurrence(qn[i:i + 1], kn[i:i + 1], v[i:i + 1], gg[i:i + 1], beta[i:i + 1], est[s],
                                      dk ** -0.5, HV // H)
        o[i] = oo[0]
    exp = O.gated_rmsnorm(O.bf16(o).reshape(-1, dk), norm_w, qkvz[:, C:].reshape(-1, dk), 1e-6, O.bf16).reshape(B, -1)
    close(y, exp, n_ulp=2, atol=1e-4, max_frac=0.05)
    torch.testing.assert_close(sd.cpu(), est, rtol=1e-4, atol=1e-5)


def test_kv_grow(K):
    g = gen(9)
    S, old, new, nkv, d = 3, 64, 192, 4, 256
    src_k = bf(torch.randn(S * old + 64, nkv, d, generator=g))
    src_v = bf(torch.randn(S * old + 64, nkv, d, generator=g))
    lengths = [10, 0, 64]
    dk_, dv_ = (torch.full((S * new + 64, nkv, d), 7.0, dtype=torch.bfloat16, device=DEV) for _ in range(2))
    K.kv_grow(src_k.to(DEV), src_v.to(DEV), dk_, dv_, torch.tensor(lengths, dtype=torch.int32, device=DEV), S, old, new)
    exp_k = torch.zeros(S * new + 64, nkv, d, dtype=torch.bfloat16)
    exp_v = torch.zeros_like(exp_k)
    for s, L in enumerate(lengths):
        exp_k[64 + s * new:64 + s * new + L] = src_k[64 + s * old:64 + s * old + L]
        exp_v[64 + s * new:64 + s * new + L] = src_v[64 + s * old:64 + s * old + L]
    assert torch.equal(dk_.cpu(), exp_k)
    assert torch.equal(dv_.cpu(), exp_v)


def test_no_device_error_after_ops(K):
    from qwen38_inference_b200 import _lib
    assert _lib.take_device_error() == 0


@pytest.mark.parametrize("M", [2, 37, 130, 300, 512])
@pytest.mark.parametrize("nq,nkv,d,rd", [(24, 4, 256, 64), (6, 1, 256, 64), (4, 2, 64, 16)])
def test_gemm_qkv_rope_store_matches_unfused(K, M, nq, nkv, d, rd):
    """The attention projection with q/k norm, RoPE and the KV store in the GEMM (or its
    split-K finisher) against the GEMM followed by qk_norm_rope_store (tested against the
    oracle above), on NaN-poisoned caches: the gate columns and the V rows bit for bit (the
    same GEMM and rounding), q and the K rows within two bf16 ulps of the larger of the
    element and its head row's RMS (the sum of squares is reduced in another order in the
    GEMM epilogue, which can move both normalized elements of a rotated pair by an ulp), no
    other cache row written. M = 2 and
    37 take the weight-streaming split-K path, 130 and 300 the one-CTA kernel or a split-K
    product where the tiles leave SMs idle, 512 a split-K chunk; d = 64 runs the GEMM and
    qk_norm_rope_store. The CTA-pair variants are compared with the one-CTA kernel below."""
    from qwen38_inference_b200.config import rope_table, HybridConfig
    g = torch.Generator(device=DEV).manual_seed(M + nq)
    H = 5120 if nq == 24 else 512
    N = (2 * nq + 2 * nkv) * d
    cfg = HybridConfig(hidden_size=64, intermediate_size=64, num_attention_heads=nq, num_key_value_heads=nkv,
                       head_dim=d, linear_num_key_heads=1, linear_num_value_heads=1, linear_key_head_dim=128,
                       linear_value_head_dim=128, linear_conv_kernel_dim=4, num_hidden_layers=4, vocab_size=8,
                       partial_rotary_factor=rd / d)
    rope = rope_table(cfg, 4096, DEV)
    x = torch.randn(M, H, device=DEV, generator=g).bfloat16()
    w = (torch.randn(N, H, device=DEV, generator=g) * 0.02).bfloat16()
    qw = (torch.randn(d, device=DEV, generator=g) * 0.1).bfloat16()
    kw = (torch.randn(d, device=DEV, generator=g) * 0.1).bfloat16()
    rows = 2 * M + 64
    pos = torch.randint(0, 4096, (M,), device=DEV, generator=g, dtype=torch.int32)
    loc = (torch.randperm(rows - 64, device=DEV, generator=g)[:M] + 64).to(torch.int32)
    ld = N + 16  # a row stride wider than the projection, as the engine's shared buffer
    caches = [torch.full((rows, nkv, d), float("nan"), dtype=torch.bfloat16, device=DEV) for _ in range(4)]
    ws = K.Workspace(DEV)
    a = torch.zeros(M, ld, dtype=torch.bfloat16, device=DEV)[:, :N]
    K.gemm_qkv_rope_store(x, w, a, nq, nkv, d, qw, kw, rope, pos, loc, caches[0], caches[1], 1e-6, ws)
    b = torch.zeros(M, ld, dtype=torch.bfloat16, device=DEV)[:, :N]
    K.gemm(x, w, b, ws=ws)
    K.qk_norm_rope_store(b, nq, nkv, d, qw, kw, rope, pos, loc, caches[2], caches[3], 1e-6)
    torch.cuda.synchronize()
    qa, qb = a[:, :2 * nq * d].reshape(M, nq, 2, d), b[:, :2 * nq * d].reshape(M, nq, 2, d)
    assert torch.equal(qa[:, :, 1], qb[:, :, 1])  # gates
    close_rows(qa[:, :, 0], qb[:, :, 0], n_ulp=2, max_frac=0.02)
    li = loc.long()
    assert torch.equal(caches[1][li], caches[3][li])  # v rows
    close_rows(caches[0][li], caches[2][li], n_ulp=2, max_frac=0.02)
    untouched = torch.ones(rows, dtype=torch.bool, device=DEV)
    untouched[li] = False
    assert bool(torch.isnan(caches[0][untouched].float()).all()) and bool(torch.isnan(caches[1][untouched].float()).all())
    from qwen38_inference_b200 import _lib
    assert _lib.take_device_error() == 0


@pytest.mark.parametrize("M", [2000, 4096])
@pytest.mark.parametrize("nq,nkv", [(24, 4), (6, 1)])
def test_gemm_qkv_rope_store_kernel_variants_agree(K, monkeypatch, M, nq, nkv):
    """The attention projection on the one-CTA kernel (the default), the CTA pair
    (QW_GEMM_PAIR=1) and its 256 x 512 tile (two head segments per unit, QW_GEMM_WIDE=4):
    projection, q/k norm and RoPE, gate and the cache rows bit for bit, on NaN-poisoned
    caches. M = 2000 is a ragged last row tile; (6, 1) at M = 2000 has too few tiles and takes
    the split-K product in every mode."""
    from qwen38_inference_b200.config import rope_table, HybridConfig
    d, rd = 256, 64
    g = torch.Generator(device=DEV).manual_seed(M * 3 + nq)
    H, N = 5120, (2 * nq + 2 * nkv) * d
    cfg = HybridConfig(hidden_size=64, intermediate_size=64, num_attention_heads=nq, num_key_value_heads=nkv,
                       head_dim=d, linear_num_key_heads=1, linear_num_value_heads=1, linear_key_head_dim=128,
                       linear_value_head_dim=128, linear_conv_kernel_dim=4, num_hidden_layers=4, vocab_size=8,
                       partial_rotary_factor=rd / d)
    rope = rope_table(cfg, 4096, DEV)
    x = torch.randn(M, H, device=DEV, generator=g).bfloat16()
    w = (torch.randn(N, H, device=DEV, generator=g) * 0.02).bfloat16()
    qw = (torch.randn(d, device=DEV, generator=g) * 0.1).bfloat16()
    kw = (torch.randn(d, device=DEV, generator=g) * 0.1).bfloat16()
    rows = 2 * M + 64
    pos = torch.randint(0, 4096, (M,), device=DEV, generator=g, dtype=torch.int32)
    loc = (torch.randperm(rows - 64, device=DEV, generator=g)[:M] + 64).to(torch.int32)
    ws = K.Workspace(DEV)
    outs = []
    for pair, mode in (("0", "0"), ("1", "0"), ("1", "4")):
        monkeypatch.setenv("QW_GEMM_PAIR", pair)
        monkeypatch.setenv("QW_GEMM_WIDE", mode)
        a = torch.zeros(M, N, dtype=torch.bfloat16, device=DEV)
        kc = torch.full((rows, nkv, d), float("nan"), dtype=torch.bfloat16, device=DEV)
        vc = torch.full((rows, nkv, d), float("nan"), dtype=torch.bfloat16, device=DEV)
        K.gemm_qkv_rope_store(x, w, a, nq, nkv, d, qw, kw, rope, pos, loc, kc, vc, 1e-6, ws)
        outs.append((a, kc, vc))
    torch.cuda.synchronize()
    for other in outs[1:]:
        for t0, t1 in zip(outs[0], other):
            assert torch.equal(t0.view(torch.int16), t1.view(torch.int16))
    from qwen38_inference_b200 import _lib
    assert _lib.take_device_error() == 0


def _ulps(got, exp, d_head):
    """|got - exp| in bf16 ulps of max(|element|, RMS of its head's d values): an output that
    cancellation in sum_s p_s v_s made small is measured at its row's scale."""
    got, exp = got.float().cpu(), exp.float().cpu()
    d = (got - exp).abs()
    rms = exp.view(exp.shape[0], -1, d_head).pow(2).mean(-1, keepdim=True).sqrt().expand(-1, -1, d_head)
    scale = torch.maximum(torch.maximum(got.abs(), exp.abs()), rms.reshape(exp.shape))
    return d / ulp(scale), d


@pytest.mark.parametrize("nq,nkv,d,case", [(24, 4, 256, "mixed"), (6, 1, 256, "mixed"), (4, 2, 64, "mixed"),
                                           (24, 4, 256, "long"), (4, 2, 64, "long")])
def test_attn_prefill_against_kernel_restatement(K, nq, nkv, d, case):
    """The prefill kernel against the CPU restatement of its own steps (64-key blocks, the
    running maximum raised only past 8, P rounded to bf16 at that scale;
    oracle/attention_kernels.py): what is left is the order of the fp32 sums and the
    hardware 2^x, at most 4 bf16 ulps at the scale of the element's head row and at most 1 %
    of the elements (measured on B200: at most 3 ulps, 0.05-0.09 % of the elements differ)."""
    from oracle import attention_kernels as AK
    from qwen38_inference_b200.model import build_metadata
    g = gen(4)
    if case == "mixed":
        prefixes, lens = [0, 37, 130, 0], [200, 1, 77, 129]
    else:
        prefixes, lens = [0, 300], [700, 260]
    kc, vc, qkv, starts = _attn_case(g, nq, nkv, d, prefixes, lens, cap=1024)
    if case == "long":
        pos = torch.arange(kc.shape[0], dtype=torch.float32).view(-1, 1, 1)
        kc = bf(kc.float() * (1.0 + pos / 256.0))
    packed, offs, T = build_metadata(list(range(len(lens))), prefixes, lens, 1024)
    md = {k: torch.from_numpy(packed[o:o + n]).to(DEV) for k, (o, n) in offs.items()}
    out = torch.empty(T, nq * d, dtype=torch.bfloat16, device=DEV)
    K.attn_prefill(qkv.to(DEV), nq, nkv, d, kc.to(DEV), vc.to(DEV), md["tiles"], md["cu"], md["prefix"],
                   md["kv_base"], out, d ** -0.5)
    exp = AK.attn_prefill(qkv.float(), nq, nkv, d, kc.float(), vc.float(), starts, prefixes, lens, d ** -0.5)
    u, diff = _ulps(out, exp, d)
    print(f"prefill {case} nq={nq}: max {u.max().item():.2f} ulp, {(diff > 0).float().mean().item():.4f} differ")
    assert u.max().item() <= 4.0 and (diff > 0).float().mean().item() <= 0.01


@pytest.mark.parametrize("nq,nkv,d", [(24, 4, 256), (4, 2, 64)])
@pytest.mark.parametrize("splits", [1, 3])
def test_attn_decode_against_kernel_restatement(K, nq, nkv, d, splits):
    """The split-KV decode kernel and its merge against the CPU restatement of their steps
    (16-key steps in two warp halves per split, exact running maximum, bf16 P, fp32 merges;
    oracle/attention_kernels.py): at most 4 bf16 ulps at the scale of the element's head row
    and at most 1 % of the elements (measured on B200: at most 2 ulps, 0.08-0.15 %)."""
    from oracle import attention_kernels as AK
    g = gen(5)
    lens = [1] * 5
    prefixes = [1, 63, 64, 300, 511]
    kc, vc, qkv, starts = _attn_case(g, nq, nkv, d, prefixes, lens)
    B = len(lens)
    seq_len = torch.tensor([p + 1 for p in prefixes], dtype=torch.int32)
    kv_base = torch.tensor(starts, dtype=torch.int32)
    out = torch.empty(B, nq * d, dtype=torch.bfloat16, device=DEV)
    K.attn_decode(qkv.to(DEV), B, nq, nkv, d, kc.to(DEV), vc.to(DEV), seq_len.to(DEV), kv_base.to(DEV), 512, splits,
                  out, d ** -0.5, K.Workspace(DEV))
    exp = AK.attn_decode(qkv.float(), nq, nkv, d, kc.float(), vc.float(), starts, [p + 1 for p in prefixes], 512,
                         splits, d ** -0.5)
    u, diff = _ulps(out, exp, d)
    print(f"decode splits={splits} nq={nq}: max {u.max().item():.2f} ulp, {(diff > 0).float().mean().item():.4f} differ")
    assert u.max().item() <= 4.0 and (diff > 0).float().mean().item() <= 0.01


def test_kv_grow_layers(K):
    """The growth of several layers' pools in one launch equals the one-layer growth of each
    (two row widths: the 27B's 4 KV heads of 256, and one head of 64, the generic path)."""
    for nkv, d in ((4, 256), (1, 64)):
        g = gen(11 + d)
        S, old, new, n_layers = 3, 64, 192, 3
        lengths = torch.tensor([10, 0, 64], dtype=torch.int32, device=DEV)
        src = [tuple(bf(torch.randn(S * old + 64, nkv, d, generator=g)).to(DEV) for _ in range(2))
               for _ in range(n_layers)]
        dst = [tuple(torch.full((S * new + 64, nkv, d), 7.0, dtype=torch.bfloat16, device=DEV) for _ in range(2))
               for _ in range(n_layers)]
        K.kv_grow_layers(src, dst, lengths, S, old, new)
        for (sk, sv), (dk, dv) in zip(src, dst):
            ek, ev = (torch.full_like(dk, 7.0) for _ in range(2))
            K.kv_grow(sk, sv, ek, ev, lengths, S, old, new)
            torch.cuda.synchronize()
            assert torch.equal(dk, ek) and torch.equal(dv, ev)
            assert torch.equal(dk[64 + 2 * new:64 + 2 * new + 64], sk[64 + 2 * old:64 + 3 * old])
