"""Python layer API, mirroring torch-ext/fp8linear/layers.py of the reference.

Same public names and contracts:
  * fake (meta) implementations so ``torch.compile`` traces through the ops
    (layers.py:11-66 of the reference);
  * ``quantize_weight`` / ``fp8_linear`` wrappers (layers.py:107-118);
  * ``quantize_(module)``: in-place e4m3 weight quantization of every eligible
    ``nn.Linear`` (layers.py:120-142);
  * ``Fp8Linear``: the stateless kernels-hub layer whose ``forward`` is grafted onto
    a quantized ``nn.Linear`` (layers.py:145-167).

Differences from the reference: ``fp8_linear`` returns ``x.dtype`` (the reference
returns fp16 and ``Fp8Linear.forward`` casts back); ``fp8_gemm`` returns bf16; the
MXFP8 path (``quantize_mxfp8``, ``quantize_weight_mxfp8``, ``mxfp8_gemm``,
``mxfp8_linear``, and ``fp8_linear`` on uint8 block scales with an e4m3 weight) and the
NVFP4 path (``quantize_nvfp4``, ``quantize_weight_nvfp4``, ``nvfp4_gemm``,
``nvfp4_linear``, and ``fp8_linear`` on uint8 block scales with a packed uint8 weight) are
implemented; ``mxfp8_gemm`` / ``nvfp4_gemm`` return bf16 and the linears ``x.dtype``.
"""
from __future__ import annotations

import torch
from torch import nn

from ._ops import add_op_namespace_prefix, ops

E4M3_MAX = 448.0


@torch.library.register_fake(add_op_namespace_prefix("fp8_linear"))
def _fp8_linear_fake(x, wq, w_scale, bias=None):
    return x.new_empty((*x.shape[:-1], wq.shape[0]), dtype=x.dtype)


@torch.library.register_fake(add_op_namespace_prefix("quantize_fp8"))
def _quantize_fp8_fake(x):
    xq = x.new_empty(x.shape, dtype=torch.float8_e4m3fn)
    scale = x.new_empty((x.shape[0],), dtype=torch.float32)
    return xq, scale


@torch.library.register_fake(add_op_namespace_prefix("quantize_weight"))
def _quantize_weight_fake(weight):
    wq = weight.new_empty(weight.shape, dtype=torch.float8_e4m3fn)
    scale = weight.new_empty((weight.shape[0],), dtype=torch.float32)
    return wq, scale


@torch.library.register_fake(add_op_namespace_prefix("fp8_gemm"))
def _fp8_gemm_fake(xq, x_scale, wq, w_scale, bias=None):
    return xq.new_empty((xq.shape[0], wq.shape[0]), dtype=torch.bfloat16)


MX_BLOCK = 32
NV_BLOCK = 16


def mx_scale_bytes(rows: int, K: int) -> int:
    """Bytes of the MXFP8 block-scale grid: 512-byte tiles over ceil(rows/128) x
    ceil((K/32)/4) (layers.py:33-36 of the reference)."""
    return ((rows + 127) // 128) * ((K // MX_BLOCK + 3) // 4) * 512


@torch.library.register_fake(add_op_namespace_prefix("mxfp8_gemm"))
def _mxfp8_gemm_fake(xq, x_scales, wq, w_scales, bias=None):
    return xq.new_empty((xq.shape[0], wq.shape[0]), dtype=torch.bfloat16)


@torch.library.register_fake(add_op_namespace_prefix("mxfp8_linear"))
def _mxfp8_linear_fake(x, wq, w_scales, bias=None):
    return x.new_empty((*x.shape[:-1], wq.shape[0]), dtype=x.dtype)


@torch.library.register_fake(add_op_namespace_prefix("quantize_mxfp8"))
def _quantize_mxfp8_fake(x):
    xq = x.new_empty(x.shape, dtype=torch.float8_e4m3fn)
    scales = x.new_empty((mx_scale_bytes(x.shape[0], x.shape[1]),), dtype=torch.uint8)
    return xq, scales


def nv_scale_bytes(rows: int, K: int) -> int:
    """Bytes of the NVFP4 block-scale grid: 512-byte tiles over ceil(rows/128) x
    ceil((K/16)/4) (layers.py:50-56 of the reference)."""
    return ((rows + 127) // 128) * ((K // NV_BLOCK + 3) // 4) * 512


@torch.library.register_fake(add_op_namespace_prefix("quantize_nvfp4"))
def _quantize_nvfp4_fake(x):
    xq = x.new_empty((x.shape[0], x.shape[1] // 2), dtype=torch.uint8)
    scales = x.new_empty((nv_scale_bytes(x.shape[0], x.shape[1]),), dtype=torch.uint8)
    return xq, scales


@torch.library.register_fake(add_op_namespace_prefix("nvfp4_gemm"))
def _nvfp4_gemm_fake(xq, x_scales, wq, w_scales, bias=None):
    return xq.new_empty((xq.shape[0], wq.shape[0]), dtype=torch.bfloat16)


@torch.library.register_fake(add_op_namespace_prefix("nvfp4_linear"))
def _nvfp4_linear_fake(x, wq, w_scales, bias=None):
    return x.new_empty((*x.shape[:-1], wq.shape[0]), dtype=x.dtype)


def quantize_weight_mxfp8(weight: torch.Tensor):
    """MXFP8 block quantization of a ``[N, K]`` weight (offline; layers.py:72-81 of the
    reference): ``(wq e4m3 [N, K], scales uint8)`` with one e8m0 scale per 32 weights
    along K, in the tiled block-scale layout the block-scaled GEMM reads. fp32 weights
    are cast to bf16 first, as the reference does."""
    w = weight.detach()
    if w.dtype not in (torch.float16, torch.bfloat16):
        w = w.to(torch.bfloat16)
    return ops.quantize_mxfp8(w.contiguous())


def mxfp8_linear(x, wq, w_scales, bias=None):
    """MXFP8 linear (layers.py:84-86 of the reference): ``wq``/``w_scales`` from
    ``quantize_weight_mxfp8``; ``x [..., K]`` is block-quantized on the fly and multiplied
    by the block-scaled tcgen05 GEMM (scales applied inside the MMA, bias fused);
    returns ``x.dtype``."""
    return ops.mxfp8_linear(x, wq, w_scales, bias)


def quantize_weight_nvfp4(weight: torch.Tensor):
    """NVFP4 block quantization of a ``[N, K]`` weight (offline; layers.py:89-98 of the
    reference): ``(wq uint8 [N, K/2], scales uint8)``, e2m1 codes packed two per byte
    (element 2j in the low nibble) and one ue4m3 scale per 16 weights along K in the tiled
    block-scale layout. fp32 weights are cast to bf16 first, as the reference does."""
    w = weight.detach()
    if w.dtype not in (torch.float16, torch.bfloat16):
        w = w.to(torch.bfloat16)
    return ops.quantize_nvfp4(w.contiguous())


def nvfp4_linear(x, wq, w_scales, bias=None):
    """NVFP4 linear (layers.py:101-103 of the reference): ``wq``/``w_scales`` from
    ``quantize_weight_nvfp4``; ``x [..., K]`` is NVFP4-quantized on the fly and multiplied
    by the block-scaled tcgen05 e2m1 GEMM (scales inside the MMA, bias fused); returns
    ``x.dtype``."""
    return ops.nvfp4_linear(x, wq, w_scales, bias)


@torch.library.register_fake(add_op_namespace_prefix("layernorm_modulate_quantize_fp8"))
def _layernorm_modulate_quantize_fp8_fake(x, shift, scale, eps=1e-6):
    M = x.numel() // x.shape[-1]
    xq = x.new_empty((M, x.shape[-1]), dtype=torch.float8_e4m3fn)
    return xq, x.new_empty((M,), dtype=torch.float32)


@torch.library.register_fake(add_op_namespace_prefix("fp8_linear_modulated"))
def _fp8_linear_modulated_fake(x, shift, scale, wq, w_scale, bias=None, eps=1e-6):
    return x.new_empty((*x.shape[:-1], wq.shape[0]), dtype=x.dtype)


def layernorm_modulate_quantize_fp8(x, shift, scale, eps: float = 1e-6):
    """The per-token e4m3 quantizer fused into the op that precedes the linear in a FLUX /
    DiT block (AdaLayerNormZero): ``y = LayerNorm(x) * (1 + scale[b]) + shift[b]``
    (LayerNorm without affine parameters, rounded to x's dtype after each step as the
    unfused bf16 torch ops round it), quantized with ``quantize_fp8``'s rule, without ``y``
    ever being written. ``x [B, T, K]`` (or ``[M, K]`` with B dividing M), ``shift`` and
    ``scale [B, K]`` in x's dtype. Returns ``(xq e4m3 [M, K], x_scale fp32 [M])`` for
    ``fp8_gemm``; no reference counterpart (it fuses the chain that feeds
    ``Fp8Linear.forward``, layers.py:165-167 of the reference)."""
    return ops.layernorm_modulate_quantize_fp8(x, shift, scale, eps)


def fp8_linear_modulated(x, shift, scale, wq, w_scale, bias=None, eps: float = 1e-6):
    """``fp8_linear(LayerNorm(x) * (1 + scale) + shift, wq, w_scale, bias)`` with the
    modulated activations never in memory: the fused LayerNorm + modulation + quantizer,
    then the FP8 GEMM with the dequant + bias epilogue. Returns ``[..., N]`` in x's
    dtype."""
    return ops.fp8_linear_modulated(x, shift, scale, wq, w_scale, bias, eps)


def quantize_weight(weight: torch.Tensor):
    """Per-output-channel e4m3 quantization of a ``[N, K]`` CUDA weight (offline).

    Returns ``(wq e4m3 [N, K], w_scale fp32 [N])`` with the reference's arithmetic
    (csrc/quantize.cu:359-365): ``w_scale = max(amax / 448, 1e-12)`` and
    ``wq = e4m3(clamp(w / w_scale, -448, 448))``.
    """
    return ops.quantize_weight(weight)


def fp8_linear(x, wq, w_scale, bias=None):
    """FP8 linear for pre-quantized weights (``wq``/``w_scale`` from quantize_weight).

    ``x [..., K]`` bf16/fp16 -> ``[..., N]`` in ``x.dtype``: per-token e4m3
    quantization of x, tcgen05 FP8 GEMM, per-token x per-channel dequant and bias
    fused in the GEMM epilogue.
    """
    return ops.fp8_linear(x, wq, w_scale, bias)


@torch.no_grad()
def quantize_(module: nn.Module) -> int:
    """In place: quantize every eligible ``nn.Linear`` weight in ``module`` to e4m3.

    The quantized weight replaces ``linear.weight`` (as a buffer) and the per-channel
    scale is stored as ``linear.weight_scale`` -- the reference's contract
    (layers.py:120-142), eligibility ``in_features % 16 == 0``. Run it once before
    grafting ``Fp8Linear.forward`` so weights are never re-quantized per forward.
    Returns the number of layers converted.
    """
    n = 0
    for child in module.modules():
        if (
            isinstance(child, nn.Linear)
            and child.in_features % 16 == 0
            and getattr(child, "weight", None) is not None
            and child.weight.dtype != torch.float8_e4m3fn
        ):
            wq, scale = quantize_weight(child.weight.data)
            del child._parameters["weight"]
            child.register_buffer("weight", wq)
            child.register_buffer("weight_scale", scale)
            n += 1
    return n


class Fp8Linear(nn.Module):
    """Stateless kernel layer: an ``nn.Linear`` forward on FP8 tensor cores.

    No constructor and no state of its own (the kernels-hub layer contract). The
    forward is grafted onto a module already converted by ``quantize_``; it reads
    the host module's e4m3 ``weight``, fp32 ``weight_scale`` and ``bias``.
    """

    weight: torch.Tensor  # e4m3 [N, K]
    weight_scale: torch.Tensor  # fp32 [N]
    bias: torch.Tensor | None

    has_backward: bool = False
    can_torch_compile: bool = True

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        out = ops.fp8_linear(x, self.weight, self.weight_scale, self.bias)
        return out.to(x.dtype)
