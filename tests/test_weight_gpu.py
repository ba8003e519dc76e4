"""Per-channel weight quantizer on the GPU, bit-exact against the C oracle and against
the reference's own ATen expression (csrc/quantize.cu:360-364) evaluated on CUDA."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from fp8linear_b200.workloads import WORKLOADS, make_weight
from tests.helpers import bits16, codes, require_sm100, u32

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _dev():
    require_sm100()
    import fp8linear_b200  # noqa: F401


def aten_quantize_weight(weight: torch.Tensor):
    """The reference's per-channel branch, literally, in ATen on the weight's device."""
    amax = weight.detach().abs().amax(1).to(torch.float)
    scale = (amax / 448.0).clamp_min(1e-12)
    wq = (weight.to(torch.float) / scale.unsqueeze(1)).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return wq, scale


@pytest.mark.parametrize("name", ["small_cpu", "flux_qkv", "flux_fc2", "flux_linear2"])
def test_weight_matches_aten_expression(name):
    from fp8linear_b200 import ops

    wl = WORKLOADS[name]
    w, _ = make_weight(wl, gen_device="cuda")
    wq, ws = ops.quantize_weight(w)
    rq, rs = aten_quantize_weight(w)
    assert torch.equal(wq.view(torch.uint8), rq.view(torch.uint8))
    assert torch.equal(ws.view(torch.int32), rs.view(torch.int32))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_weight_vs_oracle(dtype, oracle):
    from fp8linear_b200 import ops

    g = torch.Generator().manual_seed(5)
    w = (torch.randn(96, 1040, generator=g) * torch.logspace(-4, 1, 96)[:, None]).to(dtype)
    w[3] = 0
    w[7, 5] = 448.0
    wq, ws = ops.quantize_weight(w.cuda())
    arr = w.numpy() if dtype == torch.float32 else bits16(w)
    code = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}[dtype]
    oq, osc = oracle.c_quantize_weight(arr, code, recip_scalar=True)
    assert np.array_equal(codes(wq), oq)
    assert np.array_equal(u32(ws), osc.view(np.uint32))
    # and the ATen expression agrees on the same device
    rq, rs = aten_quantize_weight(w.cuda())
    assert torch.equal(wq.view(torch.uint8), rq.view(torch.uint8))


def test_weight_nan_inf_rows():
    from fp8linear_b200 import ops

    w = torch.randn(4, 64, device="cuda")
    w[1, 3] = float("nan")
    w[2, 0] = float("inf")
    wq, ws = ops.quantize_weight(w)
    rq, rs = aten_quantize_weight(w)
    a, b = wq.float(), rq.float()
    assert torch.equal(torch.isnan(a), torch.isnan(b))
    assert torch.equal(torch.nan_to_num(a), torch.nan_to_num(b))
    assert torch.equal(torch.isnan(ws), torch.isnan(rs))
    assert torch.equal(torch.nan_to_num(ws, posinf=1.0), torch.nan_to_num(rs, posinf=1.0))


def test_weight_matches_reference_op(ref_ops):
    if ref_ops is None:
        pytest.skip("reference ops not built (oracle/_ref)")
    from fp8linear_b200 import ops

    w, _ = make_weight(WORKLOADS["flux_qkv"], gen_device="cuda")
    wq, ws = ops.quantize_weight(w)
    rq, rs = ref_ops.quantize_weight(w)
    assert torch.equal(wq.view(torch.uint8), rq.view(torch.uint8))
    assert torch.equal(ws.view(torch.int32), rs.view(torch.int32))
