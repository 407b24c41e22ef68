"""tcgen05 GEMM parity against a float64 torch reference of the same op (bf16 in, fp32
accumulation, bf16 rounding of the output).

Tolerance: an fp32 sum in a different order than any reference differs from the exact
sum by a few units of 2^-24 times the sum of |x_k w_k|, so after rounding to bf16 an
element may sit one bf16 ulp from bf16(exact) (two near cancellation). The bound per
element is 1.01 ulp_bf16(max(|exact|, |got|)) + 8 sqrt(K) 2^-24 sum_k |x_k w_k|, and at
most 1% of elements may differ from bf16(exact) at all.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def ulp_bf16(x):
    x = x.float().abs().clamp_min(2.0 ** -126)
    return torch.exp2(torch.floor(torch.log2(x)) - 7)


def fp32_sum_bound(x, w):
    K = x.shape[1]
    return 8.0 * K ** 0.5 * 2.0 ** -24 * (x.double().abs() @ w.double().abs().t())


def check_bf16(got, x, w, frac=0.01):
    ref = x.double() @ w.double().t()
    exp = ref.to(torch.bfloat16).double()
    diff = (got.double() - exp).abs()
    bound = torch.maximum(ulp_bf16(ref), ulp_bf16(got)).double() * 1.01 + fp32_sum_bound(x, w)
    bad = diff > bound
    assert not bool(bad.any()), f"{int(bad.sum())} elements beyond bound, max diff {diff.max().item()}"
    assert (diff > 0).double().mean().item() <= frac


@pytest.fixture(scope="module")
def ops():
    from qwen38_inference_b200 import ops as o
    return o


SHAPES = [
    (256, 512, 320),      # exact tiles, K tail of 64
    (300, 1000, 5120),    # ragged M and N
    (1024, 768, 256),
    (129, 96, 5120),      # the ba projection shape, M tail
    (4096, 2048, 1024),   # many tiles per CTA (persistent loop, TMEM double buffer)
    (32, 1024, 512),      # skinny: weight streaming
    (1, 96, 5120),
    (5, 5120, 6144),      # skinny split-K
    (64, 4096, 17408),
    (17, 248, 512),
    (512, 5120, 17408),   # a 512-token chunk through the down projection: split-K (80 tiles)
    (300, 5120, 6144),    # ragged M, split-K
]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_bf16(ops, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N * 13 + K)
    x = (torch.randn(M, K, device="cuda", generator=g)).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    ws = ops.Workspace("cuda")
    y = ops.gemm(x, w, ws=ws)
    torch.cuda.synchronize()
    check_bf16(y, x, w)
    from qwen38_inference_b200 import _lib
    assert _lib.take_device_error() == 0


@pytest.mark.parametrize("M,N,K", [(300, 1000, 512), (8, 2048, 1024), (2, 248320 // 64, 256)])
def test_gemm_f32_logits(ops, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    y = ops.gemm(x, w, out_kind=ops.OUT_F32_OF_BF16, ws=ops.Workspace("cuda"))
    assert y.dtype == torch.float32
    check_bf16(y, x, w)


@pytest.mark.parametrize("M,I,K", [(300, 384, 512), (128, 1024, 256), (32, 512, 1024), (3, 256, 512),
                                   (32, 17408, 5120), (7, 200, 256), (64, 2304, 512), (520, 200, 256),
                                   (2048, 1536, 640)])
def test_gemm_swiglu(ops, M, I, K):
    """SwiGLU in the epilogue: large M pairs gate and up columns in one B tile; decode
    (M <= 64) pairs 64 gate rows with their 64 up rows in one weight tile when the product
    is not split over K (17408 x 5120: the model's gate_up; I = 200: a partial last tile),
    else sums split-K partials first."""
    g = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(2 * I, K, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    y = ops.gemm(x, w, out_kind=ops.OUT_SWIGLU, ws=ops.Workspace("cuda"))
    gu = (x.double() @ w.double().t()).to(torch.bfloat16).double()
    gate, up = gu[:, :I], gu[:, I:]
    ref = gate / (1 + torch.exp(-gate)) * up
    # the rounding of g and u may flip (one ulp each), then the product rounds once more
    sb = fp32_sum_bound(x, w)
    slack = ulp_bf16(gu).double() + sb
    bound = 1.01 * ulp_bf16(ref).double() + (slack[:, :I] * up.abs() + slack[:, I:] * gate.abs()) * 1.2
    diff = (y.double() - ref.to(torch.bfloat16).double()).abs()
    assert bool((diff <= bound).all()), f"max diff {diff.max().item()}"
    assert (diff > 0).double().mean().item() <= 0.02


def test_gemm_strided_input(ops):
    g = torch.Generator(device="cuda").manual_seed(3)
    big = torch.randn(200, 1024, device="cuda", generator=g).to(torch.bfloat16)
    x = big[:, 128:128 + 512]  # row stride 1024
    w = (torch.randn(640, 512, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    y = ops.gemm(x, w)
    check_bf16(y, x, w)


def test_gemm_f32_raw_split(ops):
    """Unrounded fp32 output (a tensor-parallel rank's partial product), through the wide
    split-K path and the skinny path, within fp32 summation-order error of float64."""
    from qwen38_inference_b200 import _lib
    for M, N, K in ((512, 5120, 8704), (1, 5120, 3072), (2048, 5120, 1536)):
        g = torch.Generator(device="cuda").manual_seed(M + K)
        x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
        w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        y = ops.gemm(x, w, out_kind=ops.OUT_F32, ws=ops.Workspace("cuda"))
        torch.cuda.synchronize()
        ref = x.double() @ w.double().t()
        assert y.dtype == torch.float32
        assert bool(((y.double() - ref).abs() <= fp32_sum_bound(x, w) + 1e-30).all()), (M, N, K)
    assert _lib.take_device_error() == 0


@pytest.mark.parametrize("M,N,K", [(32, 5120, 6144), (32, 5120, 17408), (5, 1024, 512), (64, 768, 2048),
                                   (512, 5120, 17408), (512, 5120, 6144), (300, 5120, 3072)])
def test_gemm_add_rmsnorm_matches_unfused(ops, M, N, K):
    """A projection fused with the add-norm after it (decode: weight streaming; a 512-token
    chunk: split-K over idle SMs) matches the projection followed by the add-norm kernel: the
    residual bit for bit (the same partials summed in the same order), the normalized output
    within one bf16 ulp (the sum of squares is reduced in another order)."""
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    resid0 = torch.randn(M, N, device="cuda", generator=g).to(torch.bfloat16)
    nw = (torch.randn(N, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    ws = ops.Workspace("cuda")
    r_a, h_a = resid0.clone(), torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    ops.gemm_add_rmsnorm(x, w, r_a, nw, h_a, 1e-6, ws)
    r_b = resid0.clone()
    h_b = ops.gemm(x, w, ws=ws)
    check_bf16(h_b, x, w)
    ops.add_rmsnorm(h_b, r_b, nw, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(r_a, r_b)
    d = (h_a.float() - h_b.float()).abs()
    ulp = torch.exp2(torch.floor(torch.log2(h_b.float().abs().clamp_min(2.0 ** -126))) - 7)
    assert bool((d <= ulp).all()) and (d > 0).float().mean().item() < 0.01


# shapes with M >= 256 and no split over K (K of at most 15 k-blocks, or enough 128 x 256 tiles
# to fill the SMs twice): the CTA-pair path when it is selected
@pytest.mark.parametrize("M,N,K,swiglu", [(512, 1024, 512, False), (300, 1000, 512, False),
                                          (1024, 16480, 320, False), (4096, 5120, 6144, False),
                                          (520, 2 * 200, 256, True), (1024, 2 * 1536, 640, True),
                                          (300, 2 * 2304, 512, True)])
def test_gemm_kernel_variants_agree(ops, monkeypatch, M, N, K, swiglu):
    """The one-CTA kernels (the default), the CTA-pair kernel (QW_GEMM_PAIR=2 and
    QW_GEMM_PAIR_SWIGLU=1, read at every call) and its 256 x 512 tile (QW_GEMM_WIDE=7) on the
    same product: every output element accumulates the same 16-wide k-steps in the same order
    in each, so the outputs are bit-identical, ragged M and N included (a last N-half wholly
    past N)."""
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    kind = ops.OUT_SWIGLU if swiglu else ops.OUT_BF16
    ws = ops.Workspace("cuda")
    outs = []
    for pair, wide in (("0", "0"), ("2", "0"), ("2", "7")):
        monkeypatch.setenv("QW_GEMM_PAIR", pair)
        monkeypatch.setenv("QW_GEMM_PAIR_SWIGLU", "1" if pair != "0" else "0")
        monkeypatch.setenv("QW_GEMM_WIDE", wide)
        outs.append(ops.gemm(x, w, out_kind=kind, ws=ws))
    torch.cuda.synchronize()
    assert torch.equal(outs[1], outs[0]) and torch.equal(outs[2], outs[0])
    if not swiglu:
        check_bf16(outs[0], x, w)
