"""Per-token quantizer on the GPU: e4m3 codes and fp32 scales bit-exact against the
CPU oracle (oracle/fp8_oracle.c restating csrc/quantize.cu:45-73), against a full-size
torch restatement, and against the reference's own compiled kernel when present."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from fp8linear_b200.workloads import WORKLOADS, make_x
from tests.helpers import bits16, codes, require_sm100, torch_quant_ref, u32

pytestmark = pytest.mark.gpu

ALL = list(WORKLOADS)
ORACLE_ROWS = 1024  # rows checked against the scalar C oracle per workload


@pytest.fixture(scope="module", autouse=True)
def _dev():
    require_sm100()
    import fp8linear_b200  # noqa: F401


def _rows(M: int, n: int, seed: int = 0) -> np.ndarray:
    if M <= n:
        return np.arange(M)
    return np.sort(np.random.default_rng(seed).choice(M, n, replace=False))


@pytest.mark.parametrize("name", ALL)
def test_quantize_workloads_bitexact(name, oracle):
    from fp8linear_b200 import ops

    wl = WORKLOADS[name]
    x = make_x(wl, gen_device="cuda")
    xq, xs = ops.quantize_fp8(x)
    torch.cuda.synchronize()
    # full size: torch restatement on the GPU
    tq, ts = torch_quant_ref(x)
    assert torch.equal(xq.view(torch.uint8), tq.view(torch.uint8))
    assert torch.equal(xs.view(torch.int32), ts.view(torch.int32))
    # row sample: scalar C oracle
    rows = _rows(wl.M, ORACLE_ROWS)
    sel = torch.from_numpy(rows).cuda()
    oq, osc = oracle.c_quantize_rows(bits16(x[sel]), oracle.BF16)
    assert np.array_equal(codes(xq[sel]), oq)
    assert np.array_equal(u32(xs[sel]), osc.view(np.uint32))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("K", [16, 24, 40, 64, 100, 1000, 1024, 3072, 4104, 12288, 15360, 65536, 70000])
def test_quantize_shapes_vs_oracle(K, dtype, oracle):
    from fp8linear_b200 import ops

    M = 37
    g = torch.Generator(device="cpu").manual_seed(K)
    x = (torch.randn(M, K, generator=g) * torch.logspace(-3, 2, M)[:, None]).to(dtype).cuda()
    xq, xs = ops.quantize_fp8(x)
    oq, osc = oracle.c_quantize_rows(bits16(x), 0 if dtype == torch.bfloat16 else 1)
    assert np.array_equal(codes(xq), oq)
    assert np.array_equal(u32(xs), osc.view(np.uint32))


def test_quantize_edge_values(oracle):
    """Zero rows, exact 448, e4m3 midpoints, subnormals, -0.0, inf and NaN inputs."""
    from fp8linear_b200 import ops

    K = 64
    lut = oracle.e4m3_decode_lut()
    fin = lut[np.isfinite(lut)]
    mids = ((fin[:-1] + fin[1:]) / 2).astype(np.float32)
    rows = [
        np.zeros(K, np.float32),                                   # all zero -> scale 1e-12
        np.full(K, -0.0, np.float32),                              # negative zeros
        np.concatenate([[448.0], np.linspace(-448, 448, K - 1)]),  # amax exactly 448
        np.resize(np.sort(np.abs(mids))[:K], K),                   # e4m3 midpoints
        np.resize(np.array([2.0 ** -10, 3 * 2.0 ** -10, 2.0 ** -9, 448.0]), K),  # subnormals
        np.resize(np.array([np.inf, 1.0, -2.0, 0.5]), K),          # inf amax -> inv 0
        np.resize(np.array([np.nan, 1.0, -3.0, 0.25]), K),         # NaN ignored by fmaxf
        np.resize(np.array([-np.inf, np.nan, 5.0, -5.0]), K),
        np.full(K, 1e-30, np.float32),                             # tiny row (bf16 rounds)
    ]
    xf = torch.from_numpy(np.stack(rows).astype(np.float32))
    for dtype, code in ((torch.bfloat16, 0), (torch.float16, 1)):
        x = xf.to(dtype).cuda()
        xq, xs = ops.quantize_fp8(x)
        oq, osc = oracle.c_quantize_rows(bits16(x), code)
        assert np.array_equal(codes(xq), oq), dtype
        assert np.array_equal(u32(xs), osc.view(np.uint32)), dtype


@pytest.mark.parametrize("M,K", [(3000, 1024), (3000, 3072), (2000, 12288), (1000, 15360),
                                 (9000, 15360)])
def test_quantize_nonfinite_rows_among_finite(M, K, oracle):
    """Rows holding inf or NaN scattered among finite rows, at widths where a row spans 2,
    4 or 8 warps (the per-row barrier exchange) and at sizes of both pipelined forms
    (9000 x 15360 is above the register form's 256 MB threshold). Every non-finite row,
    its neighbours and a sample of the rest are checked against the oracle."""
    from fp8linear_b200 import ops

    g = torch.Generator(device="cpu").manual_seed(M + K)
    x = torch.randn(M, K, generator=g)
    bad = torch.arange(5, M, 97)
    x[bad, (bad * 31) % K] = float("inf")
    x[bad[1::2], (bad[1::2] * 17) % K] = float("nan")
    x[bad[::3], (bad[::3] * 13) % K] = float("-inf")
    x[bad[-1]] = float("nan")  # an all-NaN row
    x[bad[-2]] = 0.0           # and an all-zero row
    x = x.bfloat16().cuda()
    xq, xs = ops.quantize_fp8(x)
    torch.cuda.synchronize()
    rows = set(bad.tolist()) | set((bad + 1).clamp(max=M - 1).tolist()) | set(
        (bad - 1).tolist()) | set(_rows(M, 256, seed=K).tolist())
    sel = torch.tensor(sorted(rows), device="cuda")
    oq, osc = oracle.c_quantize_rows(bits16(x[sel]), oracle.BF16)
    assert np.array_equal(codes(xq[sel]), oq)
    assert np.array_equal(u32(xs[sel]), osc.view(np.uint32))


def test_quantize_empty_and_one_row():
    from fp8linear_b200 import ops

    x = torch.empty(0, 3072, dtype=torch.bfloat16, device="cuda")
    xq, xs = ops.quantize_fp8(x)
    assert xq.shape == (0, 3072) and xs.shape == (0,)
    x = torch.randn(1, 3072, device="cuda").bfloat16()
    xq, xs = ops.quantize_fp8(x)
    tq, ts = torch_quant_ref(x)
    assert torch.equal(xq.view(torch.uint8), tq.view(torch.uint8))


def test_quantize_strided_input():
    """A non-contiguous / offset view is made contiguous first, like the reference."""
    from fp8linear_b200 import ops

    base = torch.randn(64, 3072 + 8, device="cuda").bfloat16()
    x = base[:, 4:3076]
    xq, xs = ops.quantize_fp8(x)
    tq, ts = torch_quant_ref(x.contiguous())
    assert torch.equal(xq.view(torch.uint8), tq.view(torch.uint8))


@pytest.mark.parametrize("name", ["small_cpu", "flux_qkv", "flux_fc2", "sweep_M16"])
def test_quantize_matches_reference_kernel(name, ref_ops):
    if ref_ops is None:
        pytest.skip("reference ops not built (oracle/_ref)")
    from fp8linear_b200 import ops

    wl = WORKLOADS[name]
    x = make_x(wl, gen_device="cuda")
    xq, xs = ops.quantize_fp8(x)
    rq, rs = ref_ops.quantize_fp8(x)
    assert torch.equal(xq.view(torch.uint8), rq.view(torch.uint8))
    assert torch.equal(xs.view(torch.int32), rs.view(torch.int32))


def test_quantize_capi_matches_op(capi):
    from fp8linear_b200 import ops

    x = make_x(WORKLOADS["flux_qkv"], gen_device="cuda")
    a = ops.quantize_fp8(x)
    b = capi.quantize_fp8(x)
    assert torch.equal(a[0].view(torch.uint8), b[0].view(torch.uint8))
    assert torch.equal(a[1], b[1])


@pytest.mark.parametrize("M,K", [(2000, 15360), (1500, 10240), (3000, 7168), (700, 40960),
                                 (5000, 3072), (149, 12288), (4608, 12296), (8192, 3072),
                                 (3000, 12288), (4000, 10240), (20000, 1024)])
def test_quantize_ring_configs(M, K):
    """Inputs large enough for the streaming kernel, at widths where its shared-memory row
    ring holds 3, 4, 5, 8 or 16 rows, plus register-kernel sizes: every row still
    quantizes bit-exactly."""
    from fp8linear_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(M + K)
    x = (torch.randn(M, K, device="cuda", generator=g) *
         torch.logspace(-2, 2, M, device="cuda")[:, None]).bfloat16()
    xq, xs = ops.quantize_fp8(x)
    tq, ts = torch_quant_ref(x)
    assert torch.equal(xq.view(torch.uint8), tq.view(torch.uint8))
    assert torch.equal(xs.view(torch.int32), ts.view(torch.int32))


@pytest.mark.parametrize("K", [3072, 12288, 15360])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_quantize_nonfinite_rows_wide(K, dtype, oracle):
    """Rows with inf/NaN next to finite rows at FLUX widths: the rows spanning several
    warps exercise the CTA-wide fallback to the clamp path."""
    from fp8linear_b200 import ops

    M = 300
    g = torch.Generator().manual_seed(K)
    x = torch.randn(M, K, generator=g) * 3
    for r in range(0, M, 37):
        x[r, (r * 7) % K] = float("nan")
    for r in range(5, M, 53):
        x[r, (r * 3) % K] = float("inf") if r % 2 else -float("inf")
    x = x.to(dtype)
    xq, xs = ops.quantize_fp8(x.cuda())
    oq, osc = oracle.c_quantize_rows(bits16(x), 0 if dtype == torch.bfloat16 else 1)
    assert np.array_equal(codes(xq), oq)
    assert np.array_equal(u32(xs), osc.view(np.uint32))
