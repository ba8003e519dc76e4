"""The module path with the reference's opt-in weight formats: quantize_ under
FP8LINEAR_USE_MX / FP8LINEAR_USE_NVFP4 stores MXFP8 / NVFP4 weights (csrc/quantize.cu:344-357),
and the grafted Fp8Linear.forward reaches the block-scaled GEMMs through fp8_linear's
dispatch on the weight format (csrc/fp8_gemm.cu:203-216), giving the bits of the format's
own linear and staying close to the bf16 model."""
from __future__ import annotations

import pytest
import torch
from torch import nn

from tests.helpers import require_sm100

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _dev():
    require_sm100()
    import fp8linear_b200  # noqa: F401


@pytest.mark.parametrize("env,fmt", [("FP8LINEAR_USE_MX", "mx"), ("FP8LINEAR_USE_NVFP4", "nv")])
def test_quantize_module_block_scaled(monkeypatch, env, fmt):
    import fp8linear_b200 as f

    torch.manual_seed(0)
    model = nn.Sequential(nn.Linear(256, 512), nn.GELU(), nn.Linear(512, 128)).cuda()
    model = model.to(torch.bfloat16)
    x = torch.randn(4, 33, 256, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        ref = model(x).float()
    monkeypatch.setenv(env, "1")
    assert f.quantize_(model) == 2
    l0 = model[0]
    assert l0.weight_scale.dtype == torch.uint8
    if fmt == "nv":
        assert l0.weight.dtype == torch.uint8 and l0.weight.shape == (512, 128)
    else:
        assert l0.weight.dtype == torch.float8_e4m3fn and l0.weight.shape == (512, 256)
    for m in (model[0], model[2]):
        m.forward = f.Fp8Linear.forward.__get__(m)
    with torch.no_grad():
        out = model(x)
        h = f.fp8_linear(x, l0.weight, l0.weight_scale, l0.bias)
        direct = (f.nvfp4_linear if fmt == "nv" else f.mxfp8_linear)(x, l0.weight, l0.weight_scale,
                                                                      l0.bias)
    assert out.dtype == torch.bfloat16 and out.shape == (4, 33, 128)
    assert torch.equal(h, direct)
    rel = float((out.float() - ref).norm() / ref.norm())
    assert rel < (0.25 if fmt == "nv" else 0.1)
