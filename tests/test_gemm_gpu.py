"""tcgen05 FP8 GEMM with fused dequant + bias, on the GPU.

Outputs are checked in fp32 with max|got - ref| / max|ref| <= 1e-2 against
  * the CPU oracle (exact-sum dequant-matmul, csrc/fp8_gemm.cu:65-80 restated),
  * an fp32 torch dequant-matmul at full FLUX sizes,
  * the reference's own fp8_gemm (cuBLASLt + dequant kernel, fp16 out) when built.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from fp8linear_b200.workloads import WORKLOADS, make_weight, make_x
from tests.helpers import OUT_TOL, bits16, codes, f32, max_rel, require_sm100, torch_gemm_ref

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _dev():
    require_sm100()
    import fp8linear_b200  # noqa: F401


def _operands(M, N, K, seed=0, bias_dtype=torch.bfloat16, x_dist="normal"):
    from fp8linear_b200 import ops

    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    if x_dist == "gelu":
        x = torch.nn.functional.gelu(x)
    x = x.bfloat16().cuda()
    w = (torch.randn(N, K, generator=g) * 0.02).bfloat16().cuda()
    b = None if bias_dtype is None else (torch.randn(N, generator=g) * 0.02).to(bias_dtype).cuda()
    xq, xs = ops.quantize_fp8(x)
    wq, ws = ops.quantize_weight(w)
    return xq, xs, wq, ws, b


def _oracle_out(oracle, xq, xs, wq, ws, b):
    """Exact-sum dequant-matmul + bias in fp32 (no fp16 rounding of bias/out)."""
    bias16 = None
    out = oracle.port_gemm_dequant(codes(xq), f32(xs), codes(wq), f32(ws), None,
                                   round_out=False, acc_dtype="float64")
    if b is not None:
        out = out + f32(b)[None, :]
    return out


@pytest.mark.parametrize(
    "M,N,K",
    [(1, 8, 16), (7, 24, 48), (128, 256, 128), (129, 264, 144), (300, 520, 1040),
     (256, 1024, 1024), (1000, 3072, 3072), (64, 9216, 3072), (513, 776, 4096),
     (255, 512, 12288), (3, 1, 16), (64, 44, 1024), (200, 100, 512), (257, 1003, 256),
     (333, 384, 1024), (1000, 640, 512), (192, 3072, 3072), (256, 9216, 3072),
     (384, 1024, 3072), (500, 2048, 2048),
     # 64 < M <= 128 on the few-token kernel: narrow and wide N, ragged token rows, long K
     (65, 3072, 3072), (96, 1000, 2080), (128, 9216, 3072), (100, 21504, 3072),
     (128, 3072, 15360), (127, 136, 256)],
)
def test_gemm_shapes_vs_oracle(M, N, K, oracle):
    from fp8linear_b200 import ops

    xq, xs, wq, ws, b = _operands(M, N, K, seed=M * 7 + N)
    out = ops.fp8_gemm(xq, xs, wq, ws, b)
    assert out.dtype == torch.bfloat16 and out.shape == (M, N)
    ref = _oracle_out(oracle, xq, xs, wq, ws, b)
    err = max_rel(out.cpu(), torch.from_numpy(ref))
    assert err <= OUT_TOL, err


@pytest.mark.parametrize("M,N", [(333, 384), (200, 1152), (4608, 3456), (1000, 1280)])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16])
def test_gemm_paired_stores_edges(M, N, out_dtype, capi, oracle):
    """Output widths that are multiples of 128 but not of the 256-column tile, rows not a
    multiple of 32, both output types. 4608 x 3456 keeps 256-column pair tiles (more than
    one wave), whose last tile's second chunk pair lies past N and is not stored: the
    paired 3-D stores write exactly the [M, N] block. The others fit one wave of
    192-column tiles, stored chunk by chunk; 1000 x 1280 has a partial last tile (128 of
    its 192 columns)."""
    xq, xs, wq, ws, b = _operands(M, N, 512, seed=M + N)
    out = capi.fp8_gemm(xq, xs, wq, ws, b, out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert out.dtype == out_dtype and out.shape == (M, N)
    ref = _oracle_out(oracle, xq, xs, wq, ws, b)
    assert max_rel(out.float().cpu(), torch.from_numpy(ref)) <= OUT_TOL


@pytest.mark.parametrize("bias_dtype", [None, torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16])
def test_gemm_bias_and_out_dtypes(bias_dtype, out_dtype, capi):
    xq, xs, wq, ws, b = _operands(384, 768, 512, seed=3, bias_dtype=bias_dtype)
    out = capi.fp8_gemm(xq, xs, wq, ws, b, out_dtype=out_dtype)
    ref = torch_gemm_ref(xq, xs, wq, ws, b)
    assert out.dtype == out_dtype
    assert max_rel(out, ref) <= OUT_TOL


@pytest.mark.parametrize("name", ["flux_qkv", "flux_fc1", "flux_fc2", "flux_linear1",
                                  "flux_linear2", "sweep_M1", "sweep_M16", "sweep_M128",
                                  "sweep_M1024", "sweep_M4096", "sweep_M16384", "sweep_M65536",
                                  "flux_linear2_rank8"])
def test_gemm_workloads_vs_torch_fp32(name):
    from fp8linear_b200 import ops

    wl = WORKLOADS[name]
    x = make_x(wl, gen_device="cuda")
    w, b = make_weight(wl, gen_device="cuda")
    xq, xs = ops.quantize_fp8(x)
    wq, ws = ops.quantize_weight(w)
    out = ops.fp8_gemm(xq, xs, wq, ws, b)
    # reference in fp32 on the GPU, chunked over rows to bound memory
    step = 4096
    worst = 0.0
    for r0 in range(0, wl.M, step):
        ref = torch_gemm_ref(xq[r0:r0 + step], xs[r0:r0 + step], wq, ws, b)
        worst = max(worst, max_rel(out[r0:r0 + step], ref))
        del ref
    assert worst <= OUT_TOL, worst


@pytest.mark.parametrize("name", ["small_cpu", "flux_qkv", "flux_fc2", "sweep_M1"])
def test_gemm_matches_reference_op(name, ref_ops):
    if ref_ops is None:
        pytest.skip("reference ops not built (oracle/_ref)")
    from fp8linear_b200 import ops

    wl = WORKLOADS[name]
    x = make_x(wl, gen_device="cuda")
    w, b = make_weight(wl, gen_device="cuda")
    rq, rxs = ref_ops.quantize_fp8(x)
    rwq, rws = ref_ops.quantize_weight(w)
    ref = ref_ops.fp8_gemm(rq, rxs, rwq, rws, b)  # fp16, the reference path
    wq, ws = ops.quantize_weight(w)
    xq, xs = ops.quantize_fp8(x)
    out = ops.fp8_gemm(xq, xs, wq, ws, b)
    assert max_rel(out, ref) <= OUT_TOL


def test_gemm_errors():
    from fp8linear_b200 import ops

    xq = torch.zeros(4, 24, dtype=torch.float8_e4m3fn, device="cuda")
    wq = torch.zeros(8, 24, dtype=torch.float8_e4m3fn, device="cuda")
    s4 = torch.ones(4, device="cuda")
    s8 = torch.ones(8, device="cuda")
    with pytest.raises(RuntimeError, match="multiple of 16"):
        ops.fp8_gemm(xq, s4, wq, s8, None)
    xq = torch.zeros(4, 32, dtype=torch.float8_e4m3fn, device="cuda")
    wq = torch.zeros(8, 32, dtype=torch.float8_e4m3fn, device="cuda")
    with pytest.raises(RuntimeError, match="M entries"):
        ops.fp8_gemm(xq, s8, wq, s8, None)
    with pytest.raises(RuntimeError, match="float8_e4m3fn"):
        ops.fp8_gemm(xq.view(torch.uint8), s4, wq, s8, None)


def test_gemm_empty():
    from fp8linear_b200 import ops

    xq = torch.zeros(0, 64, dtype=torch.float8_e4m3fn, device="cuda")
    wq = torch.zeros(16, 64, dtype=torch.float8_e4m3fn, device="cuda")
    out = ops.fp8_gemm(xq, torch.ones(0, device="cuda"), wq, torch.ones(16, device="cuda"), None)
    assert out.shape == (0, 16)


def test_gemm_repeatable_and_watchdog_clear(capi):
    """Two launches give identical bits (deterministic accumulation order) and no
    bounded wait in the kernel ever ran out."""
    from fp8linear_b200 import ops

    xq, xs, wq, ws, b = _operands(1024, 2048, 3072, seed=11)
    a = ops.fp8_gemm(xq, xs, wq, ws, b)
    c = ops.fp8_gemm(xq, xs, wq, ws, b)
    assert torch.equal(a, c)
    assert capi.device_status() == 0
