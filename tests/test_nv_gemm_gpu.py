"""NVFP4 GEMM on the GPU (tcgen05 kind::mxf4nvf4.block_scale, ue4m3 scales per 16 elements
in TMEM): outputs within OUT_TOL of the exact block-scaled sum (the oracle restating
csrc/fp8_gemm.cu:352-445; the reference's own cuBLASLt call has no algorithm on B200, so
its outputs cannot be pinned), and bit-identical between the fused linear, the two-step
path, the C ABI and fp8_linear's dispatch on a packed uint8 weight."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from fp8linear_b200.workloads import WORKLOADS, make_weight, make_x
from tests.helpers import OUT_TOL, bits16, f32, max_rel, require_sm100

pytestmark = pytest.mark.gpu


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
    xq, xs = f.quantize_nvfp4(x)
    wq, ws = f.quantize_weight_nvfp4(w)
    return x, w, b, xq, xs, wq, ws


def _oracle_out(oracle, xq, xs, wq, ws, b):
    return oracle.np_nvfp4_gemm(xq.cpu().numpy(), xs.cpu().numpy(), wq.cpu().numpy(),
                                ws.cpu().numpy()) + f32(b)[None, :]


@pytest.mark.parametrize("M,N,K", [(128, 256, 256), (256, 256, 256), (64, 256, 256),
                                   (256, 512, 1024), (300, 520, 160), (1, 264, 96),
                                   (129, 1000, 2080), (512, 44, 512), (384, 768, 4096)])
def test_nv_gemm_vs_oracle(oracle, M, N, K):
    """One tile and one K-block first (both shapes), then several tiles, ragged M/N, K not a
    multiple of 256 (a partial last K-block whose missing scale tiles read as zero),
    N % 8 != 0 (direct stores), the single-CTA shape (M <= 128), long K."""
    import fp8linear_b200 as f

    x, w, b, xq, xs, wq, ws = _operands(M, N, K, seed=M + N + K)
    out = f.nvfp4_gemm(xq, xs, wq, ws, b)
    torch.cuda.synchronize()
    assert out.dtype == torch.bfloat16 and out.shape == (M, N)
    ref = _oracle_out(oracle, xq, xs, wq, ws, b)
    assert max_rel(out.cpu(), torch.from_numpy(ref)) <= OUT_TOL


def test_nv_gemm_exact_small_integers(oracle):
    """Codes and scales chosen so every product and partial sum is exact in fp32: the
    GEMM must then equal the oracle exactly before the bf16 rounding, whatever the
    accumulation order (checks nibble order, scale placement per 16-block and per row)."""
    import fp8linear_b200 as f

    M, N, K = 256, 256, 512
    g = torch.Generator(device="cuda").manual_seed(11)
    # values in {0, +-0.5, +-1, +-1.5, +-2, +-3} times a power-of-two block scale
    lv = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0], device="cuda")
    x = lv[torch.randint(0, 6, (M, K), device="cuda", generator=g)]
    x = x * (torch.randint(0, 2, (M, K), device="cuda", generator=g) * 2 - 1)
    w = lv[torch.randint(0, 6, (N, K), device="cuda", generator=g)]
    # give each 16-block an amax of 6 so that its scale is exactly 1
    x[:, ::16] = 6.0
    w[:, ::16] = -6.0
    x = x.to(torch.bfloat16)
    w = w.to(torch.bfloat16)
    xq, xs = f.quantize_nvfp4(x)
    wq, ws = f.quantize_weight_nvfp4(w)
    assert bool((xs[: (M // 128) * (K // 64) * 512] == 0x38).all())
    out = f.nvfp4_gemm(xq, xs, wq, ws, None)
    torch.cuda.synchronize()
    ref = (x.float() @ w.float().T).to(torch.bfloat16)
    assert torch.equal(out.cpu(), ref.cpu())
    o = oracle.np_nvfp4_gemm(xq.cpu().numpy(), xs.cpu().numpy(), wq.cpu().numpy(),
                             ws.cpu().numpy())
    assert np.array_equal(o, (x.float() @ w.float().T).cpu().numpy())


@pytest.mark.parametrize("name", ["flux_qkv", "flux_fc2", "sweep_M16"])
def test_nv_linear_full_size(oracle, name):
    """FLUX shapes (many tiles per CTA pair: both accumulators and their shared chunk in
    use): fused linear == quantize + GEMM bit for bit; against the oracle on sampled rows."""
    import fp8linear_b200 as f

    wl = WORKLOADS[name]
    x = make_x(wl, gen_device="cuda")
    w, b = make_weight(wl, gen_device="cuda")
    wq, ws = f.quantize_weight_nvfp4(w)
    out = f.nvfp4_linear(x, wq, ws, b)
    xq, xs = f.quantize_nvfp4(x)
    two = f.nvfp4_gemm(xq, xs, wq, ws, b)
    torch.cuda.synchronize()
    assert out.dtype == x.dtype
    assert torch.equal(out, two)
    rows = np.sort(np.random.default_rng(0).choice(wl.M, min(wl.M, 96), replace=False))
    oq, osc = oracle.np_quantize_nvfp4(bits16(x[rows]), oracle.BF16)
    ref = oracle.np_nvfp4_gemm(oq, osc, wq.cpu().numpy(), ws.cpu().numpy()) + f32(b)[None, :]
    assert max_rel(out[rows].cpu(), torch.from_numpy(ref)) <= OUT_TOL


def test_fp8_linear_dispatches_on_packed_weights(capi):
    """fp8_linear with uint8 scales and a packed uint8 weight takes the NVFP4 path
    (csrc/fp8_gemm.cu:203-209); the C ABI gives the same bits."""
    import fp8linear_b200 as f

    x, w, b, xq, xs, wq, ws = _operands(1024, 768, 512, seed=5)
    a = f.fp8_linear(x.view(2, 512, 512), wq, ws, b)
    m = f.nvfp4_linear(x, wq, ws, b)
    c = capi.nvfp4_linear(x, wq, ws, b)
    torch.cuda.synchronize()
    assert a.shape == (2, 512, 768)
    assert torch.equal(a.reshape(1024, 768), m)
    assert torch.equal(c, m)


def test_nv_quantize_weight_opt_in(monkeypatch):
    """quantize_weight stays per-channel unless FP8LINEAR_USE_NVFP4 is set; it wins over
    FP8LINEAR_USE_MX (csrc/quantize.cu:344-357)."""
    import fp8linear_b200 as f

    w = torch.randn(64, 128, device="cuda", dtype=torch.bfloat16)
    wq, ws = f.quantize_weight(w)
    assert ws.dtype == torch.float32
    monkeypatch.setenv("FP8LINEAR_USE_MX", "1")
    monkeypatch.setenv("FP8LINEAR_USE_NVFP4", "1")
    wq2, ws2 = f.quantize_weight(w)
    assert wq2.dtype == torch.uint8 and wq2.shape == (64, 64)
    r_q, r_s = f.quantize_weight_nvfp4(w)
    assert torch.equal(ws2, r_s) and torch.equal(wq2, r_q)


def test_nv_gemm_argument_checks():
    import fp8linear_b200 as f

    x, w, b, xq, xs, wq, ws = _operands(8, 16, 64)
    with pytest.raises(RuntimeError, match="wrong size"):
        f.nvfp4_gemm(xq, xs[:-16], wq, ws, b)
    with pytest.raises(RuntimeError, match="uint8"):
        f.nvfp4_gemm(xq, xs.float(), wq, ws, b)
    with pytest.raises(RuntimeError, match="K mismatch"):
        f.nvfp4_gemm(xq, xs, wq[:, :16], ws, b)
