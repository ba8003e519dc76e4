"""The C ABI library without a GPU: it loads, exports every symbol the public header
declares, and its host-side argument checks reject bad calls before touching CUDA."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "fp8linear_b200.h"
LIB = ROOT / "fp8linear_b200" / "libfp8linear_b200.so"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"FP8LIN_API\s+[\w\s\*]+?\b(fp8lin_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ("fp8lin_quantize_fp8", "fp8lin_quantize_weight", "fp8lin_fp8_gemm",
              "fp8lin_fp8_linear", "fp8lin_linear_workspace_size", "fp8lin_last_error"):
        assert s in syms


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(LIB))
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_ctypes_binding_matches_header():
    from fp8linear_b200.capi import SIGNATURES

    assert sorted(SIGNATURES) == declared_symbols()


@pytest.fixture(scope="module")
def api():
    from fp8linear_b200.capi import CApi

    return CApi()


def test_version_and_info(api):
    assert api.lib.fp8lin_abi_version() == 1
    assert b"sm_100a" in api.lib.fp8lin_build_info()


def test_workspace_size(api):
    assert api.workspace_size(0, 3072) == 0
    assert api.workspace_size(4608, 3072) == 4608 * 3072 + 4608 * 4
    assert api.workspace_size(3, 16) == 256 + 256


def test_argument_checks_without_gpu(api):
    L = api.lib
    # bad dtype
    assert L.fp8lin_quantize_fp8(None, 7, 4, 16, None, None, None) == 1
    assert "fp16 or bf16" in api.last_error()
    # negative sizes
    assert L.fp8lin_quantize_fp8(None, 0, -1, 16, None, None, None) == 1
    # M == 0 is a no-op
    assert L.fp8lin_quantize_fp8(None, 0, 0, 16, None, None, None) == 0
    assert L.fp8lin_quantize_weight(None, 2, 0, 16, None, None, None) == 0
    # K % 16 (the reference's K check, fp8_gemm.cu:154); any N is accepted
    assert L.fp8lin_fp8_gemm(None, None, None, None, None, -1, None, 0, 4, 8, 24, None) == 2
    assert "multiple of 16" in api.last_error()
    assert L.fp8lin_fp8_gemm(None, None, None, None, None, -1, None, 0, 4, 12, 32, None) == 1
    assert "null" in api.last_error()
    # null pointers with work to do
    assert L.fp8lin_fp8_gemm(None, None, None, None, None, -1, None, 0, 4, 8, 32, None) == 1
    # M == 0 GEMM is a no-op
    assert L.fp8lin_fp8_gemm(None, None, None, None, None, -1, None, 0, 0, 8, 32, None) == 0
    # bad output dtype / bias dtype
    assert L.fp8lin_fp8_gemm(None, None, None, None, None, -1, None, 2, 4, 8, 32, None) == 1
    assert L.fp8lin_fp8_gemm(None, None, None, None, ctypes.c_void_p(16), 9, None, 0, 4, 8, 32,
                             None) == 1
    # fused op: workspace too small
    assert L.fp8lin_fp8_linear(ctypes.c_void_p(256), 0, ctypes.c_void_p(256), ctypes.c_void_p(256),
                               None, -1, ctypes.c_void_p(256), 0, 4, 8, 32, ctypes.c_void_p(256),
                               16, None) == 3
    assert "workspace" in api.last_error()
    # a successful call clears the message
    assert L.fp8lin_quantize_fp8(None, 0, 0, 16, None, None, None) == 0
    assert api.last_error() == ""
