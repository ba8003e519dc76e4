"""Helpers shared by the tests: tensor <-> oracle conversions and tolerances."""
from __future__ import annotations

import numpy as np
import torch

# Output tolerance: max|got - ref| / max|ref| in fp32 (fp32-accumulate tolerance for
# bf16 outputs of the dequantized FP8 GEMM).
OUT_TOL = 1e-2


def bits16(x: torch.Tensor) -> np.ndarray:
    """bf16/fp16 tensor -> uint16 numpy bit patterns (on the CPU)."""
    return x.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def codes(q: torch.Tensor) -> np.ndarray:
    """e4m3 tensor -> uint8 codes."""
    return q.detach().contiguous().cpu().view(torch.uint8).numpy()


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def u32(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int32).numpy().view(np.uint32)


def dtype_code(dt: torch.dtype) -> int:
    return {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}[dt]


def torch_quant_ref(x: torch.Tensor):
    """Full-size restatement of the per-token quantizer in torch ops (any device).

    Same operation order as the reference kernel (csrc/quantize.cu:52-72); tensor /
    tensor division keeps it an IEEE divide. Only for inputs without NaN (torch's
    amax propagates NaN where the kernel's fmaxf ignores it).
    """
    xf = x.float()
    amax = xf.abs().amax(dim=1)
    sc = torch.clamp_min(amax / torch.full_like(amax, 448.0), 1e-12)
    inv = torch.ones_like(sc) / sc
    v = (xf * inv[:, None]).clamp(-448.0, 448.0)
    return v.to(torch.float8_e4m3fn), sc


def torch_gemm_ref(xq, xs, wq, ws, bias=None):
    """fp32 dequant-matmul on the tensors' device: ((xq @ wq^T) * xs) * ws + bias."""
    acc = xq.float() @ wq.float().T
    out = acc * xs.float()[:, None] * ws.float()[None, :]
    if bias is not None:
        out = out + bias.float()[None, :]
    return out


def max_rel(got: torch.Tensor, ref: torch.Tensor) -> float:
    got = got.float()
    ref = ref.float()
    if ref.numel() == 0:
        return 0.0
    return float((got - ref).abs().max() / ref.abs().max().clamp_min(1e-30))


def require_sm100():
    """GPU tests fail (not skip) without an sm_100 device: no silent pass."""
    assert torch.cuda.is_available(), "gpu-marked test run without a CUDA device"
    major, minor = torch.cuda.get_device_capability()
    assert major == 10, f"needs sm_100, found sm_{major}{minor}"
