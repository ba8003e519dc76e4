"""The quantizer fused into the op before the linear, on the GPU: the fused LayerNorm +
AdaLN modulation + per-token e4m3 quantizer bit for bit against the oracle (which restates
its reduction order), the fused linear against quantize + GEMM, and both against the
unfused chain a FLUX block runs (torch LayerNorm and bf16 modulation on the GPU, then
quantize_fp8 -- ours and the reference's compiled op)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from fp8linear_b200.workloads import WORKLOADS, make_weight, make_x
from tests.helpers import OUT_TOL, bits16, codes, max_rel, require_sm100

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _dev():
    require_sm100()
    import fp8linear_b200  # noqa: F401


def _mod(B, K, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    shift = (torch.randn(B, K, device="cuda", generator=g) * 0.1).to(dtype)
    scale = (torch.randn(B, K, device="cuda", generator=g) * 0.2).to(dtype)
    return shift, scale


def _unfused(x, shift, scale, eps=1e-6):
    """What a FLUX block runs without the fusion (AdaLayerNormZero in bf16)."""
    K = x.shape[-1]
    x2 = x.reshape(-1, K)
    b = torch.arange(x2.shape[0], device=x.device) // (x2.shape[0] // shift.shape[0])
    ln = torch.nn.functional.layer_norm(x2, (K,), eps=eps)
    return ln * (1 + scale)[b] + shift[b]


@pytest.mark.parametrize("M,K,B,dtype", [(1, 8, 1, torch.bfloat16), (7, 96, 7, torch.bfloat16),
                                         (129, 1032, 3, torch.float16), (300, 264, 4, torch.bfloat16),
                                         (256, 8192, 2, torch.float16), (4608, 3072, 2, torch.bfloat16),
                                         (8192, 3072, 2, torch.bfloat16), (6003, 4104, 3, torch.bfloat16),
                                         (3200, 8192, 4, torch.float16)])
def test_fused_quantizer_vs_oracle(oracle, M, K, B, dtype):
    """Every CPL variant of the kernel (K/8 chunks over 32 lanes: 1 .. 32 per lane), ragged
    chunk counts, one batch per row, fp16; inputs of 50 MB and more (several waves of
    rows), ragged, and with the longest rows."""
    import fp8linear_b200 as f

    g = torch.Generator(device="cuda").manual_seed(M + K)
    x = (torch.randn(M, K, device="cuda", generator=g) * 2 + 0.3).to(dtype)
    shift, scale = _mod(B, K, dtype, seed=K)
    xq, xs = f.layernorm_modulate_quantize_fp8(x, shift, scale)
    torch.cuda.synchronize()
    dt = oracle.BF16 if dtype == torch.bfloat16 else oracle.F16
    _, oq, osc = oracle.c_ln_modulate_quantize(bits16(x), bits16(shift), bits16(scale), 1e-6, dt)
    assert np.array_equal(xs.cpu().numpy(), osc)
    assert np.array_equal(codes(xq), oq)


def test_fused_quantizer_edge_rows(oracle):
    K = 512
    x = torch.randn(8, K)
    x[0] = 3.0                                    # constant row: variance 0
    x[1, ::2] = float("inf")
    x[2, 5] = float("nan")
    x[3] = torch.linspace(-1e-30, 1e-30, K)
    x[4] = torch.linspace(-3e38, 3e38, K)
    x[5] *= 1e4
    x = x.to(torch.bfloat16).cuda()
    shift, scale = _mod(2, K, torch.bfloat16, seed=3)
    import fp8linear_b200 as f

    xq, xs = f.layernorm_modulate_quantize_fp8(x, shift, scale, 1e-5)
    torch.cuda.synchronize()
    _, oq, osc = oracle.c_ln_modulate_quantize(bits16(x), bits16(shift), bits16(scale), 1e-5)
    assert np.array_equal(xs.cpu().numpy(), osc)
    assert np.array_equal(codes(xq), oq)


def test_fused_quantizer_edge_rows_large_input(oracle):
    """The edge rows above at the head of a 50 MB input (rows in several waves)."""
    K = 3072
    g = torch.Generator().manual_seed(9)
    x = torch.randn(8192, K, generator=g)
    x[0] = 3.0
    x[1, ::2] = float("inf")
    x[2, 5] = float("nan")
    x[3] = torch.linspace(-1e-30, 1e-30, K)
    x[4] = torch.linspace(-3e38, 3e38, K)
    x[5] *= 1e4
    x = x.to(torch.bfloat16).cuda()
    shift, scale = _mod(4, K, torch.bfloat16, seed=5)
    import fp8linear_b200 as f

    xq, xs = f.layernorm_modulate_quantize_fp8(x, shift, scale, 1e-5)
    torch.cuda.synchronize()
    _, oq, osc = oracle.c_ln_modulate_quantize(bits16(x), bits16(shift), bits16(scale), 1e-5)
    assert np.array_equal(xs.cpu().numpy(), osc)
    assert np.array_equal(codes(xq), oq)


def test_fused_linear_and_capi(capi):
    """fp8_linear_modulated == fp8_gemm of the fused quantizer's output, bit for bit; the C
    ABI gives the same bits; x [B, T, K] keeps its leading shape."""
    import fp8linear_b200 as f

    wl = WORKLOADS["flux_qkv"]
    x = make_x(wl, gen_device="cuda").view(2, wl.M // 2, wl.K)
    w, b = make_weight(wl, gen_device="cuda")
    wq, ws = f.quantize_weight(w)
    shift, scale = _mod(2, wl.K, torch.bfloat16, seed=11)
    out = f.fp8_linear_modulated(x, shift, scale, wq, ws, b)
    xq, xs = f.layernorm_modulate_quantize_fp8(x, shift, scale)
    two = f.fp8_gemm(xq, xs, wq, ws, b)
    c = capi.fp8_linear_modulated(x, shift, scale, wq, ws, b)
    cq, cs = capi.layernorm_modulate_quantize_fp8(x, shift, scale)
    torch.cuda.synchronize()
    assert out.shape == (2, wl.M // 2, wl.N) and out.dtype == torch.bfloat16
    assert torch.equal(out.reshape(wl.M, wl.N), two)
    assert torch.equal(c, two)
    assert torch.equal(cq.view(torch.uint8), xq.view(torch.uint8)) and torch.equal(cs, xs)


def test_against_unfused_chain(ref_ops):
    """Against torch's LayerNorm + bf16 modulation on the GPU followed by quantize_fp8 (ours
    and, when built, the reference's): nearly every code is equal (torch's LayerNorm reduces
    in another order and uses an approximate rsqrt); the linear outputs agree within
    OUT_TOL."""
    import fp8linear_b200 as f

    wl = WORKLOADS["flux_qkv"]
    x = make_x(wl, gen_device="cuda")
    w, b = make_weight(wl, gen_device="cuda")
    wq, ws = f.quantize_weight(w)
    shift, scale = _mod(2, wl.K, torch.bfloat16, seed=5)
    xq, xs = f.layernorm_modulate_quantize_fp8(x, shift, scale)
    y = _unfused(x, shift, scale)
    uq, us = f.quantize_fp8(y)
    agree = (xq.view(torch.uint8) == uq.view(torch.uint8)).float().mean().item()
    assert agree >= 0.999
    assert float((xs / us - 1).abs().max()) <= 2 ** -7
    fused = f.fp8_linear_modulated(x, shift, scale, wq, ws, b)
    unfused = f.fp8_linear(y, wq, ws, b)
    assert max_rel(fused.float(), unfused.float()) <= OUT_TOL
    if ref_ops is not None:
        rq, rs = ref_ops.quantize_fp8(y)
        assert torch.equal(rq.view(torch.uint8), uq.view(torch.uint8)) and torch.equal(rs, us)
        r = ref_ops.fp8_linear(y, wq, ws, b)
        assert max_rel(fused.float(), r.float()) <= OUT_TOL


def test_argument_checks():
    import fp8linear_b200 as f

    x = torch.randn(4, 64, device="cuda", dtype=torch.bfloat16)
    shift, scale = _mod(2, 64, torch.bfloat16, seed=1)
    with pytest.raises(RuntimeError, match="multiple of 8"):
        f.layernorm_modulate_quantize_fp8(x[:, :60], shift[:, :60], scale[:, :60])
    with pytest.raises(RuntimeError, match="divide"):
        f.layernorm_modulate_quantize_fp8(x[:3], shift, scale)
    with pytest.raises(RuntimeError, match="dtype"):
        f.layernorm_modulate_quantize_fp8(x, shift.float(), scale)
    with pytest.raises(RuntimeError, match="8192"):
        big = torch.zeros(2, 8200, device="cuda", dtype=torch.bfloat16)
        f.layernorm_modulate_quantize_fp8(big, big[:1], big[:1])


@pytest.mark.parametrize("M,B", [(1, 1), (16, 2), (100, 4), (128, 1)])
def test_fused_linear_few_tokens(M, B):
    """Few tokens take the split-K few-token GEMM as the quantizer's PDL dependent: the
    fused modulated linear equals quantize + GEMM bit for bit there too."""
    import fp8linear_b200 as f

    K, N = 1024, 768
    g = torch.Generator(device="cuda").manual_seed(M)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(N, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    wq, ws = f.quantize_weight(w)
    shift, scale = _mod(B, K, torch.bfloat16, seed=M + 1)
    out = f.fp8_linear_modulated(x, shift, scale, wq, ws, b)
    xq, xs = f.layernorm_modulate_quantize_fp8(x, shift, scale)
    two = f.fp8_gemm(xq, xs, wq, ws, b)
    torch.cuda.synchronize()
    assert out.shape == (M, N)
    assert torch.equal(out, two)
