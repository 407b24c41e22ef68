"""CPU restatement of the reference ``Qwen38.forward_step`` (TEST INFRASTRUCTURE ONLY).

This package is the parity oracle and the timed CPU baseline. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and the
``--impl reference`` arm) may import it, and only as the checker or the CPU baseline;
the product package never imports it and has no CPU fallback.

Pinning: the per-op functions in :mod:`oracle.ops` are checked against golden vectors
produced by running the reference's own Triton kernels (reference/qwen38_inference.py)
under the Triton CPU interpreter (``tests/golden/make_golden.py``). The reference's
third-party kernels (flashinfer chunked GDN and trtllm-gen attention, sgl_kernel norms,
cuBLAS GEMMs) cannot run in this container; for those the oracle restates the published
math and parity there is pinned only through the reference's own Triton kernels for the
same recurrence (the decode GDN step) and the math definitions.
"""
from .model import OracleModel, HybridCacheCPU, token_batch  # noqa: F401
from . import ops  # noqa: F401
