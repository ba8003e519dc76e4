"""Torch op surface without a GPU: schemas, fake (meta) implementations for
torch.compile, the Python API names, and loud failure on CPU tensors."""
from __future__ import annotations

import pytest
import torch
from torch import nn

import fp8linear_b200 as f

REFERENCE_SCHEMAS = {
    "quantize_fp8": "quantize_fp8(Tensor x) -> (Tensor, Tensor)",
    "quantize_weight": "quantize_weight(Tensor weight) -> (Tensor, Tensor)",
    "fp8_gemm": "fp8_gemm(Tensor xq, Tensor x_scale, Tensor wq, Tensor w_scale, Tensor? bias) -> Tensor",
    "fp8_linear": "fp8_linear(Tensor x, Tensor wq, Tensor w_scale, Tensor? bias) -> Tensor",
}


@pytest.mark.parametrize("name", list(REFERENCE_SCHEMAS))
def test_schemas_match_reference(name):
    schema = str(getattr(f.ops, name).default._schema)
    assert schema == "fp8linear_b200::" + REFERENCE_SCHEMAS[name]


def test_public_names():
    for n in ("ops", "layers", "Fp8Linear", "fp8_linear", "quantize_", "quantize_weight",
              "quantize_fp8", "fp8_gemm", "mxfp8_linear", "quantize_weight_mxfp8",
              "quantize_mxfp8", "mxfp8_gemm", "nvfp4_linear", "quantize_weight_nvfp4",
              "quantize_nvfp4", "nvfp4_gemm"):
        assert hasattr(f, n), n
    assert f.layers.Fp8Linear.can_torch_compile and not f.layers.Fp8Linear.has_backward


def test_fake_impls():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        x = torch.empty(2, 7, 3072, dtype=torch.bfloat16)
        wq = torch.empty(9216, 3072, dtype=torch.float8_e4m3fn)
        ws = torch.empty(9216, dtype=torch.float32)
        out = f.ops.fp8_linear(x, wq, ws, None)
        assert out.shape == (2, 7, 9216) and out.dtype == torch.bfloat16
        out16 = f.ops.fp8_linear(x.half(), wq, ws, None)
        assert out16.dtype == torch.float16
        xq, xs = f.ops.quantize_fp8(x.reshape(14, 3072))
        assert xq.shape == (14, 3072) and xq.dtype == torch.float8_e4m3fn
        assert xs.shape == (14,) and xs.dtype == torch.float32
        g = f.ops.fp8_gemm(xq, xs, wq, ws, None)
        assert g.shape == (14, 9216) and g.dtype == torch.bfloat16
        w = torch.empty(64, 32, dtype=torch.bfloat16)
        a, s = f.ops.quantize_weight(w)
        assert a.shape == (64, 32) and a.dtype == torch.float8_e4m3fn and s.shape == (64,)


def test_cpu_tensors_fail_loudly():
    """No CPU kernel and no fallback: the CUDA-only ops refuse CPU tensors."""
    x = torch.randn(4, 32, dtype=torch.bfloat16)
    with pytest.raises((RuntimeError, NotImplementedError)):
        f.quantize_fp8(x)
    lin = nn.Linear(32, 16).bfloat16()
    with pytest.raises((RuntimeError, NotImplementedError)):
        f.quantize_(lin)


def test_block_scaled_entry_points_raise():
    # the MXFP8 quantizer exists but, like every op here, has no CPU kernel
    with pytest.raises((RuntimeError, NotImplementedError)):
        f.quantize_weight_mxfp8(torch.zeros(4, 32))
    with pytest.raises((RuntimeError, NotImplementedError)):
        f.mxfp8_linear(torch.zeros(2, 32, dtype=torch.bfloat16),
                       torch.zeros(4, 32, dtype=torch.float8_e4m3fn),
                       torch.zeros(512, dtype=torch.uint8))
    with pytest.raises((RuntimeError, NotImplementedError)):
        f.quantize_weight_nvfp4(torch.zeros(4, 32))
    with pytest.raises((RuntimeError, NotImplementedError)):
        f.nvfp4_linear(torch.zeros(2, 32, dtype=torch.bfloat16),
                       torch.zeros(4, 16, dtype=torch.uint8),
                       torch.zeros(512, dtype=torch.uint8))


def test_block_scaled_fake_impls():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        x = torch.empty(300, 3072, dtype=torch.bfloat16)
        xq, xs = f.ops.quantize_nvfp4(x)
        assert xq.shape == (300, 1536) and xq.dtype == torch.uint8
        assert xs.shape == (3 * 48 * 512,) and xs.dtype == torch.uint8
        wq = torch.empty(9216, 1536, dtype=torch.uint8)
        ws = torch.empty(72 * 48 * 512, dtype=torch.uint8)
        assert f.ops.nvfp4_gemm(xq, xs, wq, ws, None).dtype == torch.bfloat16
        o = f.ops.nvfp4_linear(x.half().view(3, 100, 3072), wq, ws, None)
        assert o.shape == (3, 100, 9216) and o.dtype == torch.float16
        mq, ms = f.ops.quantize_mxfp8(x)
        assert mq.shape == (300, 3072) and ms.shape == (3 * 24 * 512,)
    assert f.layers.nv_scale_bytes(300, 3072) == 3 * 48 * 512
