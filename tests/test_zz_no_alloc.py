"""qw_attn_decode_static: the allocation-free variant of qw_attn_decode whose split-KV scratch
lives in a file-scope device array of the library. Two calls in a row must give exactly the
outputs of qw_attn_decode with a caller workspace (same kernels, same split), and requests
larger than the array are rejected on the host.

This file is collected last on purpose: it must pass both alone in a fresh process (where
its first call performs the array's address lookup) and after every other test.
"""
import pytest
import torch

QW_ERR_WORKSPACE = 4
MAX_BYTES = 8 << 20


@pytest.fixture(scope="module")
def lib():
    from qwen38_inference_b200 import _lib
    from qwen38_inference_b200.build import LIB
    if not LIB.exists():
        from qwen38_inference_b200.build import build
        build()
    return _lib


def test_static_scratch_limit_on_host(lib):
    L = lib.load()
    assert L.qw_attn_decode_static_max_bytes() == MAX_BYTES
    # B=64, nq=24, d=256, splits=64 needs ~101 MB of scratch: rejected before any launch
    need = L.qw_attn_decode_workspace_bytes(64, 24, 256, 64)
    assert need > MAX_BYTES
    rc = L.qw_attn_decode_static(None, 0, 64, 24, 4, 256, None, None, None, None, 512, 64, None, 0, 0.0625, None)
    assert rc == QW_ERR_WORKSPACE


def _case(seed, B, nq, nkv, d, cap, dev):
    g = torch.Generator().manual_seed(seed)
    rows = B * cap + 64
    kc = torch.randn(rows, nkv, d, generator=g).to(torch.bfloat16).to(dev)
    vc = torch.randn(rows, nkv, d, generator=g).to(torch.bfloat16).to(dev)
    qkv = torch.randn(B, 2 * nq * d + 2 * nkv * d, generator=g).to(torch.bfloat16).to(dev)
    seq_len = torch.randint(1, cap + 1, (B,), generator=g, dtype=torch.int32).to(dev)
    kv_base = torch.tensor([64 + b * cap for b in range(B)], dtype=torch.int32, device=dev)
    return qkv, kc, vc, seq_len, kv_base


def _run(lib, name, case, B, nq, nkv, d, cap, splits, ws=None):
    qkv, kc, vc, seq_len, kv_base = case
    out = torch.empty(B, nq * d, dtype=torch.bfloat16, device=qkv.device)
    stream = torch.cuda.current_stream().cuda_stream
    args = [qkv.data_ptr(), qkv.stride(0), B, nq, nkv, d, kc.data_ptr(), vc.data_ptr(), seq_len.data_ptr(),
            kv_base.data_ptr(), cap, splits, out.data_ptr(), out.stride(0), d ** -0.5]
    if ws is not None:
        args += [ws.data_ptr(), ws.numel()]
    lib.call(name, *args, stream)
    return out


@pytest.mark.gpu
def test_static_matches_workspace_entry_two_calls(lib):
    dev = "cuda"
    L = lib.load()
    # (B, nq, nkv, d, capacity, splits): a small 27B-geometry batch, then the B32 decode
    # shape with 8 splits (6.3 MB of scratch, close to the array's size)
    shapes = [(5, 24, 4, 256, 512, 16), (32, 24, 4, 256, 2048, 8)]
    cases = [_case(11 + i, B, nq, nkv, d, cap, dev) for i, (B, nq, nkv, d, cap, _) in enumerate(shapes)]
    # two static calls back to back on one stream, no synchronisation between them
    got = [_run(lib, "qw_attn_decode_static", c, *s) for c, s in zip(cases, shapes)]
    exp = []
    for c, (B, nq, nkv, d, cap, splits) in zip(cases, shapes):
        need = L.qw_attn_decode_workspace_bytes(B, nq, d, splits)
        assert need <= MAX_BYTES
        ws = torch.empty(need, dtype=torch.uint8, device=dev)
        exp.append(_run(lib, "qw_attn_decode", c, B, nq, nkv, d, cap, splits, ws))
    torch.cuda.synchronize()
    assert lib.take_device_error() == 0
    for g_, e_ in zip(got, exp):
        assert torch.isfinite(g_.float()).all()
        assert torch.equal(g_, e_)
