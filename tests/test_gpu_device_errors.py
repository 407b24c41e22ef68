"""Device-side failure reporting without a GPU fault: a bounded wait that runs out, the
error word it leaves, and the calls after it.

The one-shot all-reduce of ``qw_gemm_add_rmsnorm_tp`` waits (2 s at most) for every peer
rank's arrival flag. Here a single process plays rank 0 of a two-rank group whose rank 1
never runs: both "peer buffers" are zeroed local device buffers, so the flag that rank 1
would raise stays zero, the wait gives up, the kernel records QW_DEV_ERR_TIMEOUT_TP and
returns. Every access stays inside the two buffers (flags and row slots of row m < M).
"""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(M, N, K, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(M, K, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    resid = torch.randn(M, N, device=DEV, generator=g).to(torch.bfloat16)
    nw = (torch.randn(N, device=DEV, generator=g) * 0.1).to(torch.bfloat16)
    return x, w, resid, nw


def _unfused(ops, x, w, resid, nw, ws):
    r = resid.clone()
    h = ops.gemm(x, w, ws=ws)
    ops.add_rmsnorm(h, r, nw, 1e-6)
    return r, h


def test_peer_allreduce_timeout_then_clean_calls():
    from qwen38_inference_b200 import _lib, ops
    L = _lib.load()
    assert _lib.take_device_error() == 0
    M, N, K = 4, 5120, 6144
    assert ops.gemm_add_rmsnorm_kernels(M, N, K) == 1  # the add-norm (and its counters) in the GEMM
    x, w, resid, nw = _inputs(M, N, K, 3)
    ws = ops.Workspace(DEV)
    nbytes = int(L.qw_tp_buffer_bytes(N))
    bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=DEV) for _ in range(2)]
    bases = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=DEV)
    hidden = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    torch.cuda.synchronize()
    t0 = time.time()
    ops.gemm_add_rmsnorm_tp(x, w, resid.clone(), nw, hidden, 1e-6, ws, bases, 2, 0, 0)
    torch.cuda.synchronize()
    waited = time.time() - t0
    assert waited >= 1.5, f"the flag wait returned after {waited:.2f} s"
    # rank 0 raised its own flag in both buffers; rank 1's flag in buffer 0 never came
    flags0 = bufs[0][:8 * 4].view(torch.int32).cpu()
    assert int(flags0[0]) == 1 and int(flags0[1]) == 0

    # the same projection through the fused single-GPU path right after: the ticket pair
    # was released by the timed-out CTAs, so every row is normalized as usual
    r_a, h_a = resid.clone(), torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    ops.gemm_add_rmsnorm(x, w, r_a, nw, h_a, 1e-6, ws)
    r_b, h_b = _unfused(ops, x, w, resid, nw, ws)
    torch.cuda.synchronize()
    assert torch.equal(r_a, r_b)
    d = (h_a.float() - h_b.float()).abs()
    ulp = torch.exp2(torch.floor(torch.log2(h_b.float().abs().clamp_min(2.0 ** -126))) - 7)
    assert bool((d <= ulp).all())
    # the first failure is the one reported; taking it clears the word
    assert _lib.take_device_error() == 105  # QW_DEV_ERR_TIMEOUT_TP
    ops.gemm_add_rmsnorm(x, w, resid.clone(), nw, h_a, 1e-6, ws)
    assert _lib.take_device_error() == 0


def test_forward_step_reports_a_recorded_device_error():
    """The engine copies the error word to the host after every call and raises at its next
    sync point (here ``Qwen38.check_device_error``), naming the code; the word is cleared
    and later calls run normally."""
    from qwen38_inference_b200 import Qwen38, _lib, ops
    from qwen38_inference_b200.config import mini
    cfg = mini(num_layers=4, vocab=2048)
    model = Qwen38(config=cfg, seed=4, device="cuda:0", max_context=1024)
    cache = model.new_cache(2, initial_capacity=64)
    model.forward_step([[1, 2, 3], [4, 5]], cache)
    model.check_device_error()  # nothing recorded
    # a timed-out peer wait (as above) records QW_DEV_ERR_TIMEOUT_TP in the library's word
    M, N, K = 2, cfg.hidden_size, cfg.attn_out_dim
    x, w, resid, nw = _inputs(M, N, K, 5)
    L = _lib.load()
    bufs = [torch.zeros(int(L.qw_tp_buffer_bytes(N)), dtype=torch.uint8, device=DEV) for _ in range(2)]
    bases = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=DEV)
    ops.gemm_add_rmsnorm_tp(x, w, resid, nw, torch.empty(M, N, dtype=torch.bfloat16, device=DEV), 1e-6,
                            ops.Workspace(DEV), bases, 2, 0, 1)
    model.forward_step([[6], [7]], cache)
    with pytest.raises(_lib.QwError, match="QW_DEV_ERR_TIMEOUT_TP"):
        model.check_device_error()
    logits = model.forward_step([[8], [9]], cache)
    model.check_device_error()
    assert bool(torch.isfinite(logits).all()) and cache.lengths == [5, 4]
    assert _lib.take_device_error() == 0
