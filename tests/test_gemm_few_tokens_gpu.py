"""The few-token GEMM at 17 to 128 tokens (per-token e4m3: swap-AB, 128 weight rows x the
tokens per CTA, K split over a cluster whose partial tiles meet in distributed shared
memory), on the GPU against the CPU oracle (csrc/fp8_gemm.cu:65-80 restated, exact
sums), max|got - ref| / max|ref| <= 1e-2: token counts from 17 to 128 (ragged against
the 16-token padding of the MMA's N), N from a ragged 136 to 21504 (K-splits from 8 down
to 1, and two waves of CTAs at 21504), K not a multiple of the 128-byte K-block; every
bias and output type, a column block of a wider output, the fused entry point, and
repeatability."""
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


@pytest.mark.parametrize("M", [17, 32, 33, 64, 96, 127, 128])
@pytest.mark.parametrize("N,K", [(3072, 3072), (136, 1024), (1000, 2080), (9216, 3072),
                                 (3072, 12288)])
def test_few_tokens_vs_oracle(M, N, K, oracle):
    from fp8linear_b200 import ops

    _, xq, xs, wq, ws, b = _operands(M, N, K, seed=M * 31 + N + K)
    out = ops.fp8_gemm(xq, xs, wq, ws, b)
    again = ops.fp8_gemm(xq, xs, wq, ws, b)
    assert out.dtype == torch.bfloat16 and out.shape == (M, N)
    assert torch.equal(out, again)
    err = max_rel(out.float().cpu(), _oracle(oracle, xq, xs, wq, ws, b))
    assert err <= OUT_TOL, err


@pytest.mark.parametrize("M,N,K", [(48, 21504, 3072), (128, 3072, 15360), (100, 264, 144)])
def test_few_tokens_wide_and_long(M, N, K, oracle):
    from fp8linear_b200 import ops

    _, xq, xs, wq, ws, b = _operands(M, N, K, seed=M + N)
    out = ops.fp8_gemm(xq, xs, wq, ws, b)
    assert max_rel(out.float().cpu(), _oracle(oracle, xq, xs, wq, ws, b)) <= OUT_TOL


@pytest.mark.parametrize("M", [24, 128])
@pytest.mark.parametrize("bias_dtype", [None, torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16])
def test_few_tokens_bias_and_out_dtypes(M, bias_dtype, out_dtype, capi, oracle):
    _, xq, xs, wq, ws, b = _operands(M, 3072, 3072, seed=M + 9, bias_dtype=bias_dtype)
    out = capi.fp8_gemm(xq, xs, wq, ws, b, out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert out.dtype == out_dtype
    assert max_rel(out.float().cpu(), _oracle(oracle, xq, xs, wq, ws, b)) <= OUT_TOL


@pytest.mark.parametrize("M", [40, 128])
def test_few_tokens_column_block_of_wider_output(M, capi):
    """ldo > N: the block lands at its columns of each row and nothing else is written."""
    import fp8linear_b200 as f

    x, xq, xs, wq, ws, b = _operands(M, 3072, 1024, seed=M)
    s, e, total = 256, 256 + 3072, 3584
    buf = torch.full((M, total), -7.0, dtype=torch.bfloat16, device="cuda")
    capi.fp8_linear_allgather(x, wq, ws, b, [buf.data_ptr() + s * buf.element_size()], ldo=total)
    torch.cuda.synchronize()
    ref = f.fp8_linear(x, wq, ws, b)
    assert torch.equal(buf[:, s:e], ref)
    assert (buf[:, :s] == -7.0).all() and (buf[:, e:] == -7.0).all()


@pytest.mark.parametrize("M", [20, 80, 128])
def test_few_tokens_fused_equals_two_ops(M, capi):
    """fp8_linear (weights issued before the dependency wait on the quantizer) gives the
    bits of quantize_fp8 + fp8_gemm, call after call."""
    import fp8linear_b200 as f
    from fp8linear_b200 import ops

    x, xq, xs, wq, ws, b = _operands(M, 3072, 3072, seed=M + 77)
    two = ops.fp8_gemm(xq, xs, wq, ws, b)
    for _ in range(3):
        assert torch.equal(f.fp8_linear(x, wq, ws, b), two)
    assert capi.device_status() == 0


def test_few_tokens_zero_and_extreme_tokens(oracle):
    """A zero token row (scale floor), one at the e4m3 limit and tiny ones among 70
    ordinary rows: each token's output follows its own scale."""
    from fp8linear_b200 import ops

    g = torch.Generator(device="cpu").manual_seed(5)
    x = torch.randn(70, 3072, generator=g)
    x[3] = 0.0
    x[40] *= 1e4
    x[69] *= 1e-4
    x = x.bfloat16().cuda()
    w = (torch.randn(3072, 3072, generator=g) * 0.02).bfloat16().cuda()
    xq, xs = ops.quantize_fp8(x)
    wq, ws = ops.quantize_weight(w)
    out = ops.fp8_gemm(xq, xs, wq, ws, None)
    ref = _oracle(oracle, xq, xs, wq, ws, None)
    assert (out[3] == 0).all()
    for m in range(70):
        if m != 3:
            assert max_rel(out[m].float().cpu(), ref[m]) <= OUT_TOL, m
