"""The C-ABI library loads without a GPU and exports every entry point include/qw200.h
declares, with the argument counts the ctypes binding uses. No compute calls."""
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "qw200.h"


def header_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    out = {}
    for m in re.finditer(r"\b(?:int|size_t)\s+(qw_\w+)\s*\(([^)]*)\)\s*;", text):
        args = [a for a in m.group(2).split(",") if a.strip() and a.strip() != "void"]
        out[m.group(1)] = len(args)
    return out


@pytest.fixture(scope="module")
def lib():
    from qwen38_inference_b200 import _lib
    from qwen38_inference_b200.build import LIB
    if not LIB.exists():
        from qwen38_inference_b200.build import build
        build()
    return _lib.load()


def test_header_parses():
    fns = header_functions()
    assert "qw_gemm_bf16" in fns and "qw_gdn_prefill" in fns and len(fns) >= 15


def test_every_declared_symbol_is_exported(lib):
    for name in header_functions():
        assert hasattr(lib, name), f"{name} missing from libqw200.so"


def test_binding_matches_header(lib):
    from qwen38_inference_b200._lib import SIGNATURES
    fns = header_functions()
    assert set(SIGNATURES) == set(fns), set(SIGNATURES) ^ set(fns)
    for name, n in fns.items():
        assert len(SIGNATURES[name][1]) == n, f"{name}: binding has {len(SIGNATURES[name][1])} args, header {n}"


def test_host_argument_checks_without_gpu(lib):
    """Argument validation happens on the host before any launch: null pointers and bad
    sizes return QW_ERR_ARG without touching the device."""
    assert lib.qw_version() >= 1
    assert lib.qw_gemm_bf16(None, None, None, 0, 0, 0, 0, 0, 0, 0, None, 0, None) == 1
    assert lib.qw_add_rmsnorm(None, None, None, 0, 0, 1e-6, None) == 1
    assert lib.qw_gemm_workspace_bytes(4096, 4096, 4096, 0) == 0  # large M: no workspace


def test_product_has_no_cpu_fallback():
    """The product package never imports the oracle (test infrastructure)."""
    for p in (ROOT / "qwen38_inference_b200").glob("*.py"):
        src = p.read_text()
        assert "import oracle" not in src and "from oracle" not in src, p.name
