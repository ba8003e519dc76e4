"""The GEMM for at most 16 tokens (warp-level f16 MMAs on exactly converted e4m3 codes
over 16 whole weight rows per CTA, K streamed in 1024-byte stages, the eight warps'
partials summed in shared memory), on the GPU against the CPU oracle (csrc/fp8_gemm.cu:
65-80 restated, exact sums), with max|got - ref| / max|ref| <= 1e-2: ragged N (not a
multiple of the 16-row CTA tile), K not a multiple of the 128-byte box or of the stage
(2-D boxes instead of the chunk view), both token fragment widths (8 and 16), every bias
and output type, column blocks of a wider output, repeatability, the fused entry point;
and its MXFP8 form (at most 8 tokens) bit-exact with power-of-two block scales."""
from __future__ import annotations

import pytest
import torch

from tests.helpers import OUT_TOL, codes, f32, max_rel, require_sm100

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _dev():
    require_sm100()
    import fp8linear_b200  # noqa: F401


def _operands(M, N, K, seed, bias_dtype=torch.bfloat16):
    from fp8linear_b200 import ops

    g = torch.Generator(device="cpu").manual_seed(seed)
    x = (torch.randn(M, K, generator=g) *
         torch.exp2(torch.randint(-6, 6, (M, 1), generator=g).float())).bfloat16().cuda()
    w = (torch.randn(N, K, generator=g) * 0.02).bfloat16().cuda()
    b = None if bias_dtype is None else (torch.randn(N, generator=g) * 0.02).to(bias_dtype).cuda()
    xq, xs = ops.quantize_fp8(x)
    wq, ws = ops.quantize_weight(w)
    return x, xq, xs, wq, ws, b


def _oracle(oracle, xq, xs, wq, ws, b):
    out = oracle.port_gemm_dequant(codes(xq), f32(xs), codes(wq), f32(ws), None,
                                   round_out=False, acc_dtype="float64")
    if b is not None:
        out = out + f32(b)[None, :]
    return torch.from_numpy(out)


@pytest.mark.parametrize(
    "M,N,K",
    [(1, 3072, 3072), (16, 3072, 3072), (8, 17, 144), (9, 200, 2080), (5, 100, 528),
     (2, 1, 16), (16, 9216, 3072), (13, 1000, 15360), (7, 24, 48), (3, 4104, 12288),
     (12, 48, 640), (1, 21504, 3072), (16, 3072, 15360)],
)
def test_rows_shapes_vs_oracle(M, N, K, oracle):
    from fp8linear_b200 import ops

    _, xq, xs, wq, ws, b = _operands(M, N, K, seed=M * 131 + N + K)
    out = ops.fp8_gemm(xq, xs, wq, ws, b)
    assert out.dtype == torch.bfloat16 and out.shape == (M, N)
    err = max_rel(out.float().cpu(), _oracle(oracle, xq, xs, wq, ws, b))
    assert err <= OUT_TOL, err


@pytest.mark.parametrize("M", [1, 8, 9, 16])
@pytest.mark.parametrize("bias_dtype", [None, torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16])
def test_rows_bias_and_out_dtypes(M, bias_dtype, out_dtype, capi, oracle):
    _, xq, xs, wq, ws, b = _operands(M, 776, 1040, seed=M + 5, bias_dtype=bias_dtype)
    out = capi.fp8_gemm(xq, xs, wq, ws, b, out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert out.dtype == out_dtype
    assert max_rel(out.float().cpu(), _oracle(oracle, xq, xs, wq, ws, b)) <= OUT_TOL


@pytest.mark.parametrize("M", [3, 16])
def test_rows_column_block_of_wider_output(M, capi):
    """ldo > N: the block lands at its columns of each row and nothing else is written."""
    import fp8linear_b200 as f

    x, xq, xs, wq, ws, b = _operands(M, 640, 1024, seed=M)
    s, e, total = 128, 128 + 640, 1024
    buf = torch.full((M, total), -7.0, dtype=torch.bfloat16, device="cuda")
    capi.fp8_linear_allgather(x, wq, ws, b, [buf.data_ptr() + s * buf.element_size()], ldo=total)
    torch.cuda.synchronize()
    ref = f.fp8_linear(x, wq, ws, b)
    assert torch.equal(buf[:, s:e], ref)
    assert (buf[:, :s] == -7.0).all() and (buf[:, e:] == -7.0).all()


@pytest.mark.parametrize("M", [1, 6, 16])
def test_rows_fused_equals_two_ops_and_repeats(M, capi):
    """fp8_linear (weights issued before the dependency wait on the quantizer) gives the
    bits of quantize_fp8 + fp8_gemm, and every launch gives the same bits."""
    import fp8linear_b200 as f
    from fp8linear_b200 import ops

    x, xq, xs, wq, ws, b = _operands(M, 3072, 3072, seed=M + 77)
    two = ops.fp8_gemm(xq, xs, wq, ws, b)
    fused = [f.fp8_linear(x, wq, ws, b) for _ in range(3)]
    for y in fused:
        assert torch.equal(y, two)
    assert torch.equal(ops.fp8_gemm(xq, xs, wq, ws, b), two)
    assert capi.device_status() == 0


def test_rows_zero_and_extreme_tokens(oracle):
    """A zero token row (scale floor), a row at the e4m3 limit and tiny rows among
    ordinary ones: each token's output follows its own scale."""
    from fp8linear_b200 import ops

    g = torch.Generator(device="cpu").manual_seed(3)
    x = torch.randn(11, 2048, generator=g)
    x[2] = 0.0
    x[5] *= 1e4
    x[7] *= 1e-4
    x = x.bfloat16().cuda()
    w = (torch.randn(300, 2048, generator=g) * 0.02).bfloat16().cuda()
    xq, xs = ops.quantize_fp8(x)
    wq, ws = ops.quantize_weight(w)
    out = ops.fp8_gemm(xq, xs, wq, ws, None)
    ref = _oracle(oracle, xq, xs, wq, ws, None)
    assert (out[2] == 0).all()
    for m in range(11):
        if m != 2:
            assert max_rel(out[m].float().cpu(), ref[m]) <= OUT_TOL, m


def _pow2_mx_blocks(rows, K, g):
    """Integers {0, 1, 2, 3} x sign x 2^e per 32-element block (e in {0, 1}), each block
    led by +-6 x 2^e: exact in e4m3 after the MX scale 2^(e - 6), and every sum of
    products exact in fp32, so the output is the float64 product rounded once."""
    lv = torch.tensor([0.0, 1.0, 2.0, 3.0], device="cuda")
    v = lv[torch.randint(0, 4, (rows, K), device="cuda", generator=g)]
    v[:, ::32] = 6.0
    v = v * (torch.randint(0, 2, (rows, K), device="cuda", generator=g) * 2 - 1)
    e = torch.randint(0, 2, (rows, K // 32), device="cuda", generator=g).float()
    return (v * torch.exp2(e).repeat_interleave(32, dim=1)).to(torch.bfloat16)


@pytest.mark.parametrize("M", [1, 5, 8, 9, 16])
@pytest.mark.parametrize("N,K", [(520, 3072), (136, 1024), (3072, 2048)])
def test_rows_mxfp8_exact_power_of_two_scales(M, N, K):
    """MXFP8 with few tokens (M <= 8 on the warp-level kernel, 9 and 16 on the split-K
    kernel): each 32-byte K-step of the warp-level kernel is one block whose sum takes the
    weight row's and the token's scale. Scales 1 or 2 per row and block, several stages,
    weight rows in both halves and all four 32-row groups of their scale tiles, ragged N:
    a scale taken from the wrong row, token or block changes the bits."""
    import fp8linear_b200 as f

    g = torch.Generator(device="cuda").manual_seed(1000 + 7 * M + N)
    x = _pow2_mx_blocks(M, K, g)
    w = _pow2_mx_blocks(N, K, g)
    xq, xs = f.quantize_mxfp8(x)
    wq, ws = f.quantize_weight_mxfp8(w)
    out = f.mxfp8_gemm(xq, xs, wq, ws, None)
    torch.cuda.synchronize()
    ref = (x.double().cpu() @ w.double().cpu().T).float().to(torch.bfloat16)
    assert torch.equal(out.cpu(), ref)
    assert torch.equal(f.mxfp8_linear(x, wq, ws, None), out)


@pytest.mark.parametrize("M,N,K", [(1, 3072, 3072), (7, 1000, 4096), (8, 44, 8192)])
def test_rows_mxfp8_vs_oracle(oracle, M, N, K):
    """MXFP8 on the warp-level kernel on normal data against the oracle's MX product
    (csrc/fp8_gemm.cu:233-333 restated), with bias; two calls give the same bits."""
    import fp8linear_b200 as f

    gen = torch.Generator(device="cuda").manual_seed(M + N + K)
    x = torch.randn(M, K, device="cuda", generator=gen).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    b = (torch.randn(N, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    xq, xs = f.quantize_mxfp8(x)
    wq, ws = f.quantize_weight_mxfp8(w)
    out = f.mxfp8_gemm(xq, xs, wq, ws, b)
    again = f.mxfp8_gemm(xq, xs, wq, ws, b)
    torch.cuda.synchronize()
    assert torch.equal(out, again)
    ref = oracle.np_mxfp8_gemm(codes(xq), xs.cpu().numpy(), codes(wq), ws.cpu().numpy())
    ref = ref + f32(b)[None, :]
    assert max_rel(out.cpu(), torch.from_numpy(ref)) <= OUT_TOL
