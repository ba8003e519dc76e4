"""Fused fp8_linear, the Fp8Linear layer and quantize_ on the GPU."""
from __future__ import annotations

import numpy as np
import pytest
import torch
from torch import nn

from fp8linear_b200.workloads import WORKLOADS, make_weight, make_x
from tests.helpers import (OUT_TOL, bits16, codes, f32, max_rel, require_sm100,
                           torch_gemm_ref, torch_quant_ref)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _dev():
    require_sm100()
    import fp8linear_b200  # noqa: F401


def test_small_cpu_config_vs_oracle(oracle):
    """The CPU-runnable workload end to end against the full C oracle path."""
    import fp8linear_b200 as f

    wl = WORKLOADS["small_cpu"]
    x = make_x(wl)            # seeded on the CPU: oracle and GPU see identical bytes
    w, b = make_weight(wl)
    owq, ows = oracle.c_quantize_weight(bits16(w), oracle.BF16)
    oxq, oxs = oracle.c_quantize_rows(bits16(x), oracle.BF16)
    ref = oracle.c_gemm_dequant(oxq, oxs, owq, ows, None, round_out=False) + f32(b)[None, :]
    wq, ws = f.quantize_weight(w.cuda())
    assert np.array_equal(codes(wq), owq)
    assert np.array_equal(f32(ws).view(np.uint32), ows.view(np.uint32))
    out = f.fp8_linear(x.cuda(), wq, ws, b.cuda())
    assert out.dtype == torch.bfloat16
    assert max_rel(out.cpu(), torch.from_numpy(ref)) <= OUT_TOL
    # the reference's own error measure vs the unquantized bf16 linear (informational bound)
    lin = torch.nn.functional.linear(x.float(), w.float(), b.float())
    assert oracle.norm_rel_err(f32(out), lin.numpy()) < 0.1


@pytest.mark.parametrize("name", ["flux_qkv", "flux_fc1", "flux_fc2", "sweep_M1", "sweep_M128"])
def test_fp8_linear_equals_quant_then_gemm(name):
    """fp8_linear (quantizer + PDL-launched GEMM) gives the same bits as the two ops."""
    import fp8linear_b200 as f

    wl = WORKLOADS[name]
    x = make_x(wl, gen_device="cuda")
    w, b = make_weight(wl, gen_device="cuda")
    wq, ws = f.quantize_weight(w)
    out = f.fp8_linear(x, wq, ws, b)
    xq, xs = f.quantize_fp8(x)
    ref = f.fp8_gemm(xq, xs, wq, ws, b)
    assert torch.equal(out, ref)
    assert max_rel(out, torch_gemm_ref(xq, xs, wq, ws, b)) <= OUT_TOL


def test_fp8_linear_nd_input_and_fp16():
    import fp8linear_b200 as f

    x = torch.randn(2, 3, 77, 256, device="cuda")
    w = torch.randn(512, 256, device="cuda") * 0.02
    wq, ws = f.quantize_weight(w.bfloat16())
    for dt in (torch.bfloat16, torch.float16):
        out = f.fp8_linear(x.to(dt), wq, ws, None)
        assert out.shape == (2, 3, 77, 512) and out.dtype == dt
        xq, xs = torch_quant_ref(x.to(dt).reshape(-1, 256))
        ref = torch_gemm_ref(xq, xs, wq, ws).reshape(2, 3, 77, 512)
        assert max_rel(out, ref) <= OUT_TOL


def test_fp8_linear_capi_matches_op(capi):
    import fp8linear_b200 as f

    wl = WORKLOADS["flux_qkv"]
    x = make_x(wl, gen_device="cuda")
    w, b = make_weight(wl, gen_device="cuda")
    wq, ws = f.quantize_weight(w)
    assert torch.equal(capi.fp8_linear(x, wq, ws, b), f.fp8_linear(x, wq, ws, b))


def test_quantize_and_fp8linear_module():
    """quantize_ + Fp8Linear.forward grafted onto nn.Linear, the kernels-hub contract."""
    import fp8linear_b200 as f

    torch.manual_seed(0)
    model = nn.Sequential(nn.Linear(256, 512), nn.GELU(), nn.Linear(512, 128, bias=False),
                          nn.Linear(100, 8)).cuda().bfloat16()
    x = torch.randn(4, 33, 256, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        ref_out = model[2](model[1](model[0](x))).float()
    n = f.quantize_(model)
    assert n == 2  # in_features 100 is not a multiple of 16
    assert model[0].weight.dtype == torch.float8_e4m3fn and model[0].weight_scale.dtype == torch.float32
    assert model[3].weight.dtype == torch.bfloat16
    for m in (model[0], model[2]):
        m.forward = f.Fp8Linear.forward.__get__(m)
    with torch.no_grad():
        out = model[2](model[1](model[0](x)))
    assert out.dtype == torch.bfloat16 and out.shape == (4, 33, 128)
    rel = float((out.float() - ref_out).norm() / ref_out.norm())
    assert rel < 0.1


@pytest.mark.parametrize("M", [1, 16, 64, 300])
def test_fp8_linear_right_after_the_weight_writer(M):
    """The weight buffers are rewritten and the fused linear follows on the stream with no
    synchronization between them. Behind this library's per-token quantizer the
    few-token GEMMs load their first weight stages before their own dependency wait (the
    quantizer lets them launch only after its wait, so after the writer has completed),
    and they prefetch their weights into L2 early; every read must see the new codes. Each
    round rewrites the same buffers with other values (the warp-level kernel, the split-K
    kernel and the CTA pairs); the outputs must equal the ones computed after a full
    synchronize, bit for bit."""
    import fp8linear_b200 as f
    from fp8linear_b200 import ops

    g = torch.Generator(device="cpu").manual_seed(M)
    x = torch.randn(M, 3072, generator=g).bfloat16().cuda()
    ws_list = [(torch.randn(3072, 3072, generator=g) * 0.02).bfloat16().cuda() for _ in range(4)]
    b = (torch.randn(3072, generator=g) * 0.02).bfloat16().cuda()
    wq = torch.empty(3072, 3072, dtype=torch.float8_e4m3fn, device="cuda")
    wsc = torch.empty(3072, dtype=torch.float32, device="cuda")
    outs = []
    for w in ws_list:  # writer, then the linear, back to back
        q, s = ops.quantize_weight(w)
        wq.copy_(q)
        wsc.copy_(s)
        outs.append(f.fp8_linear(x, wq, wsc, b))
    torch.cuda.synchronize()
    for w, got in zip(ws_list, outs):
        q, s = ops.quantize_weight(w)
        torch.cuda.synchronize()
        ref = f.fp8_linear(x, q, s, b)
        torch.cuda.synchronize()
        assert torch.equal(got, ref)
