"""NVFP4 block quantizer on the GPU: packed e2m1 codes and the tiled ue4m3 scale grid bit
for bit against the reference's own quantize_nvfp4 outputs (golden vectors over every
positive finite bf16 and fp16 block amax, edge rows, FLUX rows), the CPU oracle (restating
csrc/quantize.cu:157-194 and :290-334) at full FLUX sizes and ragged shapes, and the
reference's compiled kernel run live when present."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from fp8linear_b200.workloads import WORKLOADS, make_weight, make_x
from tests.helpers import bits16, require_sm100

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_nv_vectors.npz"


@pytest.fixture(scope="module", autouse=True)
def _dev():
    require_sm100()
    import fp8linear_b200  # noqa: F401


def _golden_x(g, name) -> torch.Tensor:
    dt = int(g[f"{name}_dtype"])
    if f"{name}_x" in g:
        t = torch.from_numpy(np.ascontiguousarray(g[f"{name}_x"]).view(np.int16))
        return t.view(torch.bfloat16 if dt == 0 else torch.float16)
    # the sweeps are rebuilt from their definition instead of stored
    sys.path.insert(0, str(GOLDEN.parent))
    import make_golden_nv as G

    return G.sweep_rows(torch.bfloat16 if dt == 0 else torch.float16)


@pytest.mark.skipif(not GOLDEN.exists(), reason="NVFP4 golden vectors not generated")
@pytest.mark.parametrize("name", ["sweep", "sweep16", "edge", "edge16", "rows"])
def test_nv_quantize_matches_reference_vectors(name):
    import fp8linear_b200 as f

    g = np.load(GOLDEN)
    x = _golden_x(g, name).cuda()
    xq, sc = f.quantize_nvfp4(x)
    torch.cuda.synchronize()
    assert xq.dtype == torch.uint8 and xq.shape == (x.shape[0], x.shape[1] // 2)
    assert np.array_equal(sc.cpu().numpy(), g[f"{name}_scales"])
    st = int(g[f"{name}_code_stride"])
    assert np.array_equal(xq.cpu().numpy()[::st], g[f"{name}_codes"])


@pytest.mark.parametrize("name", ["flux_qkv", "flux_fc2", "sweep_M1", "sweep_M16", "small_cpu"])
def test_nv_quantize_workloads_vs_oracle(name, oracle):
    import fp8linear_b200 as f

    wl = WORKLOADS[name]
    x = make_x(wl, gen_device="cuda")
    xq, sc = f.quantize_nvfp4(x)
    torch.cuda.synchronize()
    oq, osc = oracle.np_quantize_nvfp4(bits16(x), oracle.BF16)
    assert np.array_equal(sc.cpu().numpy(), osc)
    assert np.array_equal(xq.cpu().numpy(), oq)


@pytest.mark.parametrize("M,K,dtype", [(1, 32, torch.bfloat16), (7, 96, torch.bfloat16),
                                       (129, 1056, torch.float16), (300, 2080, torch.bfloat16),
                                       (256, 4096, torch.float16), (3, 160, torch.float16)])
def test_nv_quantize_shapes_vs_oracle(oracle, M, K, dtype):
    """Ragged rows (padded row tiles), K not a multiple of 1024 (partial warp segments) and
    K/16 not a multiple of 4 (padded scale columns), rows spread over 40 binades."""
    import fp8linear_b200 as f

    g = torch.Generator(device="cuda").manual_seed(M * 31 + K)
    x = (torch.randn(M, K, device="cuda", generator=g) *
         torch.exp2(torch.randint(-20, 20, (M, 1), device="cuda", generator=g).float())).to(dtype)
    xq, sc = f.quantize_nvfp4(x)
    torch.cuda.synchronize()
    oq, osc = oracle.c_quantize_nvfp4(bits16(x), oracle.BF16 if dtype == torch.bfloat16 else oracle.F16)
    assert np.array_equal(sc.cpu().numpy(), osc)
    assert np.array_equal(xq.cpu().numpy(), oq)


def test_nv_quantize_live_reference_kernel(ref_ops):
    if ref_ops is None:
        pytest.skip("reference ops not built")
    import fp8linear_b200 as f

    for M, K in [(4608, 3072), (333, 160), (1, 64)]:
        x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
        x[0, :5] = torch.tensor([float("inf"), float("nan"), -0.0, 1e-40, 3e38])
        a_q, a_s = f.quantize_nvfp4(x)
        r_q, r_s = ref_ops.quantize_nvfp4(x)
        torch.cuda.synchronize()
        assert torch.equal(a_s, r_s)
        assert torch.equal(a_q, r_q)


def test_nv_weight_quant_and_capi(capi):
    """quantize_weight_nvfp4 is the same quantizer on weights; the C ABI writes the whole
    padded grid itself (a buffer full of junk comes back identical to the op's)."""
    import fp8linear_b200 as f

    wl = WORKLOADS["flux_qkv"]
    w, _ = make_weight(wl, gen_device="cuda")
    w = w[:200].contiguous()
    wq, ws = f.quantize_weight_nvfp4(w)
    assert wq.shape == (200, wl.K // 2)
    assert ws.numel() == capi.nv_scale_bytes(200, wl.K) == 2 * (wl.K // 16 // 4) * 512
    junk = torch.full_like(ws, 0xAA)
    q2, s2 = capi.quantize_nvfp4(w, scales=junk)
    torch.cuda.synchronize()
    assert torch.equal(s2, ws)
    assert torch.equal(q2, wq)
    # fp32 weights go through bf16 first, as the reference does
    q3, s3 = f.quantize_weight_nvfp4(w.float())
    assert torch.equal(q3, wq) and torch.equal(s3, ws)


def test_nv_quantize_rejects_bad_k(capi):
    import fp8linear_b200 as f

    x = torch.randn(4, 48, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="multiple of 32"):
        f.quantize_nvfp4(x)
    with pytest.raises(RuntimeError, match="multiple of 32"):
        capi.quantize_nvfp4(x)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_nv_quantize_nonfinite_segments_among_finite(oracle, dtype):
    """inf and NaN in a few 1024-element segments of a 3000 x 3072 input (three segments
    per row, several segments per warp of the persistent grid, the next one in flight):
    segments with NaN take the literal clamp, the others the fast conversion, and both
    must give the oracle's codes and scales for every row."""
    import fp8linear_b200 as f

    g = torch.Generator(device="cpu").manual_seed(11)
    x = torch.randn(3000, 3072, generator=g)
    rows = torch.arange(3, 3000, 131)
    x[rows, (rows * 37) % 3072] = float("nan")
    x[rows[::2] + 1, (rows[::2] * 53) % 3072] = float("inf")
    x[rows[1::3] + 2, (rows[1::3] * 7) % 3072] = float("-inf")
    x[rows[-1]] = float("nan")
    x = x.to(dtype).cuda()
    xq, sc = f.quantize_nvfp4(x)
    torch.cuda.synchronize()
    oq, osc = oracle.np_quantize_nvfp4(bits16(x), oracle.BF16 if dtype == torch.bfloat16 else oracle.F16)
    assert np.array_equal(sc.cpu().numpy(), osc)
    assert np.array_equal(xq.cpu().numpy(), oq)
