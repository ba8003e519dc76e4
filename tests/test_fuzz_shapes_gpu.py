"""Seeded random shapes through every GEMM dispatch path, on the GPU.

The fixed grids of the other GPU tests pin each kernel's edges; this file draws shapes
across all of them at once so that a shape between the grids' points (a token count
that lands on another kernel, a K-split the heuristic has not been tested with, a
ragged N on the direct-store path) is covered too. Per shape: the output within
max|got - ref| / max|ref| <= 1e-2 of the dequant-matmul (per-token e4m3: fp32 torch
on the device, which sums the exactly decoded codes; MXFP8 / NVFP4: the oracle's
float64 block-scaled product, csrc/fp8_gemm.cu:233-333 and 352-445 restated), two
calls bit-identical, and the fused linear bit-identical to quantizer + GEMM.

Token counts are drawn per bucket of the dispatcher: 1-16 (warp-level kernel), 17-128
(split-K few-token kernel), 129-256 (few-token kernel with two token blocks, or CTA
pairs when it gets no K-split), 257-3000 (CTA pairs, 192- or 256-column tiles).

The other entry points get random shapes too: the host-buffer linear and the
no-allocation linear must give the device linear's bits, and the fused LayerNorm +
modulation quantizer the oracle's codes and scales (with its linear equal to quantizer
+ GEMM).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.helpers import OUT_TOL, f32, max_rel, require_sm100, torch_gemm_ref

pytestmark = pytest.mark.gpu

M_BUCKETS = [(1, 16), (17, 128), (129, 256), (257, 3000)]


@pytest.fixture(scope="module", autouse=True)
def _dev():
    require_sm100()
    import fp8linear_b200  # noqa: F401

    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False  # the fp32 reference sums in fp32
    yield
    torch.backends.cuda.matmul.allow_tf32 = tf32


def _draw(seed: int, count: int, k_mult: int, k_max: int, m_max: int):
    """`count` shapes (M, N, K), the token buckets in turn; N a multiple of 8 three times
    in four (TMA stores), else any width (direct stores); K log-uniform, k_mult | K."""
    rng = np.random.default_rng(seed)
    shapes = []
    for i in range(count):
        lo, hi = M_BUCKETS[i % len(M_BUCKETS)]
        M = int(rng.integers(lo, min(hi, m_max) + 1))
        if rng.random() < 0.75:
            N = 8 * int(rng.integers(1, 513))
        else:
            N = int(rng.integers(1, 700))
        K = k_mult * max(1, int(round(np.exp(rng.uniform(0, np.log(k_max / k_mult))))))
        shapes.append((M, N, K))
    return shapes


E4M3_SHAPES = _draw(seed=2024, count=40, k_mult=16, k_max=8192, m_max=3000)
MX_SHAPES = _draw(seed=7, count=16, k_mult=32, k_max=4096, m_max=1200)
NV_SHAPES = _draw(seed=11, count=16, k_mult=32, k_max=4096, m_max=1200)


def _x_w_b(M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = (torch.randn(M, K, device="cuda", generator=g) *
         torch.exp2(torch.randint(-4, 4, (M, 1), device="cuda", generator=g).float()))
    w = torch.randn(N, K, device="cuda", generator=g) * 0.02
    b = torch.randn(N, device="cuda", generator=g) * 0.02
    return x.bfloat16(), w.bfloat16(), b.bfloat16()


@pytest.mark.parametrize("M,N,K", E4M3_SHAPES)
def test_fuzz_fp8_gemm(M, N, K):
    import fp8linear_b200 as f
    from fp8linear_b200 import ops

    x, w, b = _x_w_b(M, N, K, seed=M * 7919 + N * 31 + K)
    xq, xs = ops.quantize_fp8(x)
    wq, ws = ops.quantize_weight(w)
    out = ops.fp8_gemm(xq, xs, wq, ws, b)
    assert out.shape == (M, N) and out.dtype == torch.bfloat16
    assert torch.equal(ops.fp8_gemm(xq, xs, wq, ws, b), out)
    assert torch.equal(f.fp8_linear(x, wq, ws, b), out)
    err = max_rel(out, torch_gemm_ref(xq, xs, wq, ws, b))
    assert err <= OUT_TOL, err


@pytest.mark.parametrize("M,N,K", MX_SHAPES)
def test_fuzz_mxfp8_gemm(M, N, K, oracle):
    import fp8linear_b200 as f

    x, w, b = _x_w_b(M, N, K, seed=M * 131 + N + K)
    xq, xs = f.quantize_mxfp8(x)
    wq, ws = f.quantize_weight_mxfp8(w)
    out = f.mxfp8_gemm(xq, xs, wq, ws, b)
    assert out.shape == (M, N)
    assert torch.equal(f.mxfp8_gemm(xq, xs, wq, ws, b), out)
    assert torch.equal(f.mxfp8_linear(x, wq, ws, b), out)
    ref = oracle.np_mxfp8_gemm(xq.cpu().view(torch.uint8).numpy(), xs.cpu().numpy(),
                               wq.cpu().view(torch.uint8).numpy(), ws.cpu().numpy())
    ref = ref + f32(b)[None, :]
    assert max_rel(out.cpu(), torch.from_numpy(ref)) <= OUT_TOL


@pytest.mark.parametrize("M,N,K", NV_SHAPES)
def test_fuzz_nvfp4_gemm(M, N, K, oracle):
    import fp8linear_b200 as f

    x, w, b = _x_w_b(M, N, K, seed=M * 17 + N + K)
    xq, xs = f.quantize_nvfp4(x)
    wq, ws = f.quantize_weight_nvfp4(w)
    out = f.nvfp4_gemm(xq, xs, wq, ws, b)
    assert out.shape == (M, N)
    assert torch.equal(f.nvfp4_gemm(xq, xs, wq, ws, b), out)
    assert torch.equal(f.nvfp4_linear(x, wq, ws, b), out)
    ref = oracle.np_nvfp4_gemm(xq.cpu().numpy(), xs.cpu().numpy(), wq.cpu().numpy(),
                               ws.cpu().numpy()) + f32(b)[None, :]
    assert max_rel(out.cpu(), torch.from_numpy(ref)) <= OUT_TOL


def _draw_rows(seed: int, count: int, m_max: int, k_mult: int, k_max: int, n_max: int):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(count):
        M = int(np.exp(rng.uniform(0, np.log(m_max))))
        K = k_mult * int(rng.integers(1, k_max // k_mult + 1))
        N = 8 * int(rng.integers(1, n_max // 8 + 1))
        out.append((M, N, K))
    return out


HOST_SHAPES = _draw_rows(seed=3, count=10, m_max=5000, k_mult=16, k_max=4096, n_max=2048)
NOALLOC_SHAPES = _draw_rows(seed=5, count=8, m_max=4000, k_mult=16, k_max=4096, n_max=2048)
MOD_SHAPES = _draw_rows(seed=13, count=12, m_max=2000, k_mult=16, k_max=8192, n_max=1024)


@pytest.mark.parametrize("M,N,K", HOST_SHAPES)
def test_fuzz_host_entry_point(M, N, K, capi):
    """fp8lin_fp8_linear_host (row chunks of 512 whose upload, kernels and download
    overlap) gives the device path's bits; x in bf16 or fp16."""
    from fp8linear_b200 import ops

    dtype = torch.float16 if (M + N) % 2 else torch.bfloat16
    x, w, b = _x_w_b(M, N, K, seed=M + 3 * N + K)
    x, w, b = x.to(dtype), w.to(dtype), b.to(dtype)
    wq, ws = ops.quantize_weight(w)
    want = capi.fp8_linear(x, wq, ws, b)
    got = capi.fp8_linear_host(x.cpu().pin_memory(), wq, ws, b)
    torch.cuda.current_stream().synchronize()
    assert got.dtype == dtype and torch.equal(got, want.cpu())


@pytest.mark.parametrize("M,N,K", NOALLOC_SHAPES)
def test_fuzz_noalloc_entry_point(M, N, K, capi):
    """fp8lin_fp8_linear_noalloc (the library's fixed scratch array) gives the bits of
    fp8lin_fp8_linear (a caller workspace), shape after shape on one scratch."""
    from fp8linear_b200 import ops

    x, w, b = _x_w_b(M, N, K, seed=M + N + 5 * K)
    wq, ws = ops.quantize_weight(w)
    got = capi.fp8_linear_noalloc(x, wq, ws, b)
    want = capi.fp8_linear(x, wq, ws, b)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


@pytest.mark.parametrize("M,N,K", MOD_SHAPES)
def test_fuzz_modulated(M, N, K, oracle, capi):
    """LayerNorm + modulation + quantizer bit for bit against the oracle (codes and
    scales), for 1 to 4 batches of rows, bf16 or fp16; the fused linear (out in x's
    dtype) equal to quantizer + GEMM with that output type."""
    import fp8linear_b200 as f
    from tests.helpers import bits16, codes

    B = 1 + (M + K) % 4
    M = max(B, M - M % B)  # whole batches of rows
    dtype = torch.float16 if K % 32 else torch.bfloat16
    g = torch.Generator(device="cuda").manual_seed(M * 3 + K)
    x = (torch.randn(M, K, device="cuda", generator=g) * 1.5 + 0.2).to(dtype)
    shift = (torch.randn(B, K, device="cuda", generator=g) * 0.1).to(dtype)
    scale = (torch.randn(B, K, device="cuda", generator=g) * 0.2).to(dtype)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(dtype)
    wq, ws = f.quantize_weight(w)
    xq, xs = f.layernorm_modulate_quantize_fp8(x, shift, scale)
    out = f.fp8_linear_modulated(x, shift, scale, wq, ws, None)
    two = capi.fp8_gemm(xq, xs, wq, ws, None, out_dtype=dtype)
    torch.cuda.synchronize()
    assert out.dtype == dtype and torch.equal(out, two)
    dt = oracle.BF16 if dtype == torch.bfloat16 else oracle.F16
    _, oq, osc = oracle.c_ln_modulate_quantize(bits16(x), bits16(shift), bits16(scale), 1e-6, dt)
    assert np.array_equal(xs.cpu().numpy(), osc)
    assert np.array_equal(codes(xq), oq)
