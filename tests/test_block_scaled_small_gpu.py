"""MXFP8 and NVFP4 GEMMs for few tokens (M <= 128, and two 128-token blocks up to 256) on
the GPU: the split-K swap-AB kernel with the weight's scale tiles as the MMA's scale A and
the tokens' as its scale B. Exact
against a float64 product when every scale is a power of two and every sum is exact in
fp32 (so a scale tile or TMEM column out of place changes the bits); within OUT_TOL of the
oracle (restating csrc/fp8_gemm.cu:233-333 and 352-445) on normal data; the fused linear
equal to quantize + GEMM bit for bit; repeated calls deterministic."""
from __future__ import annotations

import pytest
import torch

from tests.helpers import OUT_TOL, codes, f32, max_rel, require_sm100

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _dev():
    require_sm100()
    import fp8linear_b200  # noqa: F401


def _ops(fmt):
    import fp8linear_b200 as f

    if fmt == "mx":
        return f.quantize_mxfp8, f.quantize_weight_mxfp8, f.mxfp8_gemm, f.mxfp8_linear
    return f.quantize_nvfp4, f.quantize_weight_nvfp4, f.nvfp4_gemm, f.nvfp4_linear


def _pow2_blocks(rows, K, block, g):
    """Integers {0, 1, 2, 3} x sign x 2^e, e in {0, 1} per (row, block), each block led by
    +-6 x 2^e: the block amax is 6 x 2^e, so the MX scale is 2^(e-6) and the NV scale 2^e,
    and every value is exact in e4m3 / e2m1 after scaling."""
    lv = torch.tensor([0.0, 1.0, 2.0, 3.0], device="cuda")
    v = lv[torch.randint(0, 4, (rows, K), device="cuda", generator=g)]
    v[:, ::block] = 6.0
    v = v * (torch.randint(0, 2, (rows, K), device="cuda", generator=g) * 2 - 1)
    e = torch.randint(0, 2, (rows, K // block), device="cuda", generator=g).float()
    return (v * torch.exp2(e).repeat_interleave(block, dim=1)).to(torch.bfloat16)


@pytest.mark.parametrize("fmt", ["mx", "nv"])
@pytest.mark.parametrize("M", [1, 16, 37, 128, 200, 256, 384, 500, 513])
def test_exact_power_of_two_scales(fmt, M):
    """Per-row, per-block scales 1 or 2 on both operands: products and partial sums are
    integers of a few thousand, exact in fp32 in any summation order, so the output is the
    exact product rounded once to bf16, and a scale applied to the wrong row or block
    changes it. M = 200 and 256 use two token blocks (the second block's rows and scale
    tiles from row 128); M = 384, 500 and 513 check the CTA-pair kernel the same way."""
    qx, qw, gemm, _ = _ops(fmt)
    N, K = 384, 1024
    block = 32 if fmt == "mx" else 16
    g = torch.Generator(device="cuda").manual_seed(100 + M)
    x = _pow2_blocks(M, K, block, g)
    w = _pow2_blocks(N, K, block, g)
    xq, xs = qx(x)
    wq, ws = qw(w)
    out = gemm(xq, xs, wq, ws, None)
    torch.cuda.synchronize()
    ref = (x.double().cpu() @ w.double().cpu().T).float().to(torch.bfloat16)
    assert torch.equal(out.cpu(), ref)


def _normal(M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(N, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    return x, w, b


@pytest.mark.parametrize("fmt", ["mx", "nv"])
@pytest.mark.parametrize("M,N,K", [(1, 3072, 3072), (5, 1000, 2080), (64, 264, 96),
                                   (100, 520, 512), (128, 384, 8192), (16, 44, 4096)])
def test_vs_oracle(oracle, fmt, M, N, K):
    """Normal data: the weight-streaming shape, ragged N and K (a partial last K-block whose
    missing scale tiles read as zero), one K-block (split 1), long K (8 K-splits), N % 8 != 0;
    two calls give the same bits (fixed-order cluster reduction)."""
    qx, qw, gemm, _ = _ops(fmt)
    x, w, b = _normal(M, N, K, seed=M + N + K)
    xq, xs = qx(x)
    wq, ws = qw(w)
    out = gemm(xq, xs, wq, ws, b)
    again = gemm(xq, xs, wq, ws, b)
    torch.cuda.synchronize()
    assert out.dtype == torch.bfloat16 and out.shape == (M, N)
    assert torch.equal(out, again)
    if fmt == "mx":
        ref = oracle.np_mxfp8_gemm(codes(xq), xs.cpu().numpy(), codes(wq), ws.cpu().numpy())
    else:
        ref = oracle.np_nvfp4_gemm(xq.cpu().numpy(), xs.cpu().numpy(), wq.cpu().numpy(),
                                   ws.cpu().numpy())
    ref = ref + f32(b)[None, :]
    assert max_rel(out.cpu(), torch.from_numpy(ref)) <= OUT_TOL


@pytest.mark.parametrize("fmt", ["mx", "nv"])
@pytest.mark.parametrize("M", [1, 16, 100, 128, 200, 256, 384])
def test_linear_equals_quantize_then_gemm(fmt, M):
    """The fused linear (GEMM launched as the quantizer's programmatic dependent, weight
    tiles requested before the dependency wait) gives the two-step path's bits."""
    qx, qw, gemm, linear = _ops(fmt)
    x, w, b = _normal(M, 3072, 3072, seed=7 * M)
    wq, ws = qw(w)
    out = linear(x, wq, ws, b)
    xq, xs = qx(x)
    two = gemm(xq, xs, wq, ws, b)
    torch.cuda.synchronize()
    assert torch.equal(out, two)
