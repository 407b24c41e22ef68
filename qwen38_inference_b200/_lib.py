"""ctypes binding of ``libqw200.so`` (the C ABI declared in include/qw200.h).

Loading never falls back: a missing or unloadable library raises ImportError, and every
nonzero status from an entry point raises :class:`QwError`.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libqw200.so"

P = C.c_void_p
I32 = C.c_int
I64 = C.c_int64
SZ = C.c_size_t
F32 = C.c_float

ERRORS = {1: "QW_ERR_ARG", 2: "QW_ERR_ALIGN", 3: "QW_ERR_UNSUPPORTED", 4: "QW_ERR_WORKSPACE", 5: "QW_ERR_DRIVER"}
# values of the device error word (include/qw200.h QW_DEV_ERR_*)
DEVICE_ERRORS = {101: "QW_DEV_ERR_TIMEOUT_GEMM", 102: "QW_DEV_ERR_INDEX", 103: "QW_DEV_ERR_TIMEOUT_GDN",
                 104: "QW_DEV_ERR_TIMEOUT_ATTN", 105: "QW_DEV_ERR_TIMEOUT_TP", 106: "QW_DEV_ERR_GEMM_COUNTER"}


def device_error_name(code: int) -> str:
    return DEVICE_ERRORS.get(code, f"device error {code}")

# name -> (restype, argtypes); kept in the order of include/qw200.h
SIGNATURES = {
    "qw_version": (I32, []),
    "qw_take_device_error": (I32, [C.POINTER(I32)]),
    "qw_peek_device_error_async": (I32, [P, P]),
    "qw_gemm_workspace_bytes": (SZ, [I64, I64, I64, I32]),
    "qw_gemm_bf16": (I32, [P, P, P, I64, I64, I64, I64, I64, I64, I32, P, SZ, P]),
    "qw_gemm_add_rmsnorm_workspace_bytes": (SZ, [I64, I64, I64]),
    "qw_gemm_add_rmsnorm_kernels": (I32, [I64, I64, I64]),
    "qw_gemm_add_rmsnorm": (I32, [P, P, I64, I64, I64, I64, I64, P, P, P, F32, P, SZ, P]),
    "qw_add_rmsnorm_f32": (I32, [P, I64, I64, I64, I64, P, P, P, F32, P]),
    "qw_round_f32_bf16": (I32, [P, P, I64, P]),
    "qw_gather_vocab_shards": (I32, [P, I64, I64, I64, P, P]),
    "qw_tp_buffer_bytes": (SZ, [I64]),
    "qw_ipc_alloc": (I32, [SZ, C.POINTER(C.c_void_p), P]),
    "qw_ipc_open": (I32, [P, C.POINTER(C.c_void_p)]),
    "qw_ipc_close": (I32, [P]),
    "qw_ipc_free": (I32, [P]),
    "qw_gemm_add_rmsnorm_tp": (I32, [P, P, I64, I64, I64, I64, I64, P, P, P, F32, P, SZ, P, I64, I64, I64, I64, P]),
    "qw_embed_rmsnorm": (I32, [P, I64, P, I64, I64, P, P, P, F32, P]),
    "qw_add_rmsnorm": (I32, [P, P, P, I64, I64, F32, P]),
    "qw_add_rmsnorm_rows": (I32, [P, P, P, I64, I64, I64, P, P, F32, P]),
    "qw_gated_rmsnorm": (I32, [P, I64, P, I64, P, P, I64, I64, I64, I64, F32, P]),
    "qw_qk_norm_rope_store": (I32, [P, I64, I64, I64, I64, I64, P, P, P, I64, I64, P, P, P, P, I64, F32, P]),
    "qw_gemm_qkv_workspace_bytes": (SZ, [I64, I64, I64, I64, I64]),
    "qw_gemm_qkv_rope_store": (I32, [P, P, P, I64, I64, I64, I64, I64, I64, I64, I64, I64, P, P, P, I64, I64, P, P, P,
                                     P, I64, F32, P, SZ, P]),
    "qw_attn_prefill": (I32, [P, I64, I64, I64, I64, P, P, P, I64, P, P, P, P, I64, F32, I64, I64, P]),
    "qw_attn_prefill_split_workspace_bytes": (SZ, [I64, I64, I64, I64]),
    "qw_attn_prefill_split": (I32, [P, I64, I64, I64, I64, P, P, P, I64, P, P, P, P, I64, F32, I64, I64, I64, P, SZ, P]),
    "qw_attn_decode_workspace_bytes": (SZ, [I64, I64, I64, I64]),
    "qw_attn_decode": (I32, [P, I64, I64, I64, I64, I64, P, P, P, P, I64, I64, P, I64, F32, P, SZ, P]),
    "qw_attn_decode_static_max_bytes": (SZ, []),
    "qw_attn_decode_static": (I32, [P, I64, I64, I64, I64, I64, P, P, P, P, I64, I64, P, I64, F32, P]),
    "qw_conv_prefill": (I32, [P, I64, P, P, P, P, P, I64, I64, I64, P, P, P, I64, I64, I64, P]),
    "qw_gdn_prefill": (I32, [P, P, P, P, I64, P, P, P, P, I64, I64, I64, P, P, I64, P, P, I64, I64, I64, I64, I64,
                             F32, F32, P]),
    "qw_gdn_decode": (I32, [P, I64, P, I64, P, P, P, P, I64, I64, P, P, P, P, I64, I64, I64, I64, I64, F32, P]),
    "qw_kv_grow": (I32, [P, P, P, P, P, I64, I64, I64, I64, P]),
    "qw_kv_grow_layers": (I32, [P, P, P, P, I64, P, I64, I64, I64, I64, P]),
}


class QwError(RuntimeError):
    pass


_lib = None


def load():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is not built; run `python -m qwen38_inference_b200.build`")
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        name = ERRORS.get(rc) or (f"cudaError {rc - 1000}" if rc >= 1000 else str(rc))
        raise QwError(f"{what} failed: {name}")


# When set to a list, every entry-point call appends (name, start_event, end_event) recorded
# on the current stream around it (the benchmark's per-op breakdown).
PROFILE = None


def call(name: str, *args) -> None:
    prof = PROFILE
    if prof is None:
        check(getattr(load(), name)(*args), name)
        return
    import torch
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    check(getattr(load(), name)(*args), name)
    e1.record()
    prof.append((name, e0, e1))


def take_device_error() -> int:
    code = I32(0)
    check(load().qw_take_device_error(C.byref(code)), "qw_take_device_error")
    return code.value
