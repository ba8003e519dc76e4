"""fp8linear_b200 -- B200 (sm_100a) fused FP8 linear with drbh/fp8linear's op surface.

Public names follow torch-ext/fp8linear/__init__.py of the reference. The ops live
in ``torch.ops.fp8linear_b200`` and run hand-written sm_100a CUDA kernels through
the C ABI in ``libfp8linear_b200.so`` (include/fp8linear_b200.h).
"""
from . import layers
from ._ops import ops
from .layers import (
    Fp8Linear,
    fp8_linear,
    fp8_linear_modulated,
    layernorm_modulate_quantize_fp8,
    mxfp8_linear,
    nvfp4_linear,
    quantize_,
    quantize_weight,
    quantize_weight_mxfp8,
    quantize_weight_nvfp4,
)

quantize_fp8 = ops.quantize_fp8
fp8_gemm = ops.fp8_gemm
quantize_mxfp8 = ops.quantize_mxfp8
mxfp8_gemm = ops.mxfp8_gemm
quantize_nvfp4 = ops.quantize_nvfp4
nvfp4_gemm = ops.nvfp4_gemm

__all__ = [
    "ops",
    "layers",
    "Fp8Linear",
    "fp8_linear",
    "quantize_",
    "quantize_weight",
    "quantize_fp8",
    "fp8_gemm",
    "mxfp8_linear",
    "quantize_weight_mxfp8",
    "quantize_mxfp8",
    "mxfp8_gemm",
    "nvfp4_linear",
    "quantize_weight_nvfp4",
    "quantize_nvfp4",
    "nvfp4_gemm",
    "layernorm_modulate_quantize_fp8",
    "fp8_linear_modulated",
]
