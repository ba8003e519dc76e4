"""MXFP8 GEMM on the GPU (tcgen05 kind::mxf8f6f4.block_scale, e8m0 scales in TMEM):
outputs within OUT_TOL of the exact block-scaled sum (the oracle restating
csrc/fp8_gemm.cu:233-333), of the reference's own cuBLASLt output (golden vectors and,
when built, its compiled op run live), and bit-identical between the fused linear, the
two-step path, the C ABI and fp8_linear's dispatch on uint8 scales."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from fp8linear_b200.workloads import WORKLOADS, make_weight, make_x
from tests.helpers import OUT_TOL, bits16, codes, f32, max_rel, require_sm100

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_mx_vectors.npz"


@pytest.fixture(scope="module", autouse=True)
def _dev():
    require_sm100()
    import fp8linear_b200  # noqa: F401


def _operands(M, N, K, seed=0, dtype=torch.bfloat16):
    import fp8linear_b200 as f

    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, K, device="cuda", generator=g).to(dtype)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(dtype)
    b = (torch.randn(N, device="cuda", generator=g) * 0.02).to(dtype)
    xq, xs = f.quantize_mxfp8(x)
    wq, ws = f.quantize_weight_mxfp8(w)
    return x, w, b, xq, xs, wq, ws


def _oracle_out(oracle, xq, xs, wq, ws, b):
    return oracle.np_mxfp8_gemm(codes(xq), xs.cpu().numpy(), codes(wq), ws.cpu().numpy()) + \
        f32(b)[None, :]


@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (64, 256, 128), (256, 512, 1024),
                                   (300, 520, 160), (1, 264, 96), (129, 1000, 2080),
                                   (512, 44, 256)])
def test_mx_gemm_vs_oracle(oracle, M, N, K):
    """One tile and one K-block first, then several tiles, ragged M/N, K not a multiple of
    128 (a partial last K-block with padded scales), N % 8 != 0 (direct stores), the
    single-CTA shape (M <= 128)."""
    import fp8linear_b200 as f

    x, w, b, xq, xs, wq, ws = _operands(M, N, K, seed=M + N + K)
    out = f.mxfp8_gemm(xq, xs, wq, ws, b)
    torch.cuda.synchronize()
    assert out.dtype == torch.bfloat16 and out.shape == (M, N)
    ref = _oracle_out(oracle, xq, xs, wq, ws, b)
    assert max_rel(out.cpu(), torch.from_numpy(ref)) <= OUT_TOL


@pytest.mark.skipif(not GOLDEN.exists(), reason="MX golden vectors not generated")
def test_mx_gemm_matches_reference_vectors():
    import fp8linear_b200 as f

    g = np.load(GOLDEN)
    xq = torch.from_numpy(g["rows_codes"]).view(torch.float8_e4m3fn).cuda()
    xs = torch.from_numpy(g["rows_scales"]).cuda()
    wq = torch.from_numpy(g["gemm_wq"]).view(torch.float8_e4m3fn).cuda()
    ws = torch.from_numpy(g["gemm_ws"]).cuda()
    b = torch.from_numpy(g["gemm_b"].view(np.int16)).view(torch.bfloat16).cuda()
    out = f.mxfp8_gemm(xq, xs, wq, ws, b)
    ref = torch.from_numpy(g["gemm_out_f16"].view(np.float16).astype(np.float32))
    assert max_rel(out.cpu(), ref) <= OUT_TOL


@pytest.mark.parametrize("name", ["flux_qkv", "flux_fc2", "sweep_M16"])
def test_mx_linear_full_size(oracle, ref_ops, name):
    """FLUX shapes (many tiles per CTA pair: both accumulators and their shared chunk in
    use): fused linear == quantize + GEMM bit for bit; against the oracle on sampled rows;
    against the reference's cuBLASLt MXFP8 GEMM when built (it has no kernel for M = 16)."""
    import fp8linear_b200 as f

    wl = WORKLOADS[name]
    x = make_x(wl, gen_device="cuda")
    w, b = make_weight(wl, gen_device="cuda")
    wq, ws = f.quantize_weight_mxfp8(w)
    out = f.mxfp8_linear(x, wq, ws, b)
    xq, xs = f.quantize_mxfp8(x)
    two = f.mxfp8_gemm(xq, xs, wq, ws, b)
    torch.cuda.synchronize()
    assert out.dtype == x.dtype
    assert torch.equal(out, two)
    rows = np.sort(np.random.default_rng(0).choice(wl.M, min(wl.M, 96), replace=False))
    oq, osc = oracle.np_quantize_mxfp8(bits16(x[rows]), oracle.BF16)
    ref = oracle.np_mxfp8_gemm(oq, osc, codes(wq), ws.cpu().numpy()) + f32(b)[None, :]
    assert max_rel(out[rows].cpu(), torch.from_numpy(ref)) <= OUT_TOL
    if ref_ops is not None and wl.M > 128:
        r = ref_ops.mxfp8_gemm(xq, xs, wq, ws, b)
        assert max_rel(out.float(), r.float()) <= OUT_TOL


def test_fp8_linear_dispatches_on_block_scales(capi):
    """fp8_linear with uint8 scales takes the MXFP8 path (csrc/fp8_gemm.cu:206-213); the
    C ABI gives the same bits."""
    import fp8linear_b200 as f

    x, w, b, xq, xs, wq, ws = _operands(1024, 768, 512, seed=5)
    a = f.fp8_linear(x.view(2, 512, 512), wq, ws, b)
    m = f.mxfp8_linear(x, wq, ws, b)
    c = capi.mxfp8_linear(x, wq, ws, b)
    torch.cuda.synchronize()
    assert a.shape == (2, 512, 768)
    assert torch.equal(a.reshape(1024, 768), m)
    assert torch.equal(c, m)


def test_mx_quantize_weight_opt_in(monkeypatch):
    """quantize_weight stays per-channel unless FP8LINEAR_USE_MX is set (the reference's
    opt-in, csrc/quantize.cu:344-357)."""
    import fp8linear_b200 as f

    w = torch.randn(64, 128, device="cuda", dtype=torch.bfloat16)
    wq, ws = f.quantize_weight(w)
    assert ws.dtype == torch.float32
    monkeypatch.setenv("FP8LINEAR_USE_MX", "1")
    wq2, ws2 = f.quantize_weight(w)
    assert ws2.dtype == torch.uint8
    r_q, r_s = f.quantize_weight_mxfp8(w)
    assert torch.equal(ws2, r_s) and torch.equal(wq2.view(torch.uint8), r_q.view(torch.uint8))


def test_mx_gemm_argument_checks():
    import fp8linear_b200 as f

    x, w, b, xq, xs, wq, ws = _operands(8, 16, 64)
    with pytest.raises(RuntimeError, match="wrong size"):
        f.mxfp8_gemm(xq, xs[:-16], wq, ws, b)
    with pytest.raises(RuntimeError, match="uint8"):
        f.mxfp8_gemm(xq, xs.float(), wq, ws, b)
