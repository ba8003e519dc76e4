"""MXFP8 and NVFP4 linears with fp16 activations (fp16 out, the epilogue's other store
type), fp32 and absent bias, on both kernel shapes (single CTAs for M <= 128, CTA pairs
above), against the oracle's exact block-scaled sums; and the C ABI GEMMs writing fp16."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.helpers import OUT_TOL, codes, f32, max_rel, require_sm100

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _dev():
    require_sm100()
    import fp8linear_b200  # noqa: F401


def _case(M, N, K, seed, bias_dtype):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.float16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.float16)
    b = None if bias_dtype is None else (torch.randn(N, device="cuda", generator=g) * 0.02).to(bias_dtype)
    return x, w, b


@pytest.mark.parametrize("fmt", ["mx", "nv"])
@pytest.mark.parametrize("M,N,K,bias_dtype", [(64, 264, 256, torch.float32), (300, 520, 512, None),
                                              (129, 256, 1024, torch.float32),
                                              (333, 384, 512, torch.bfloat16), (300, 640, 1024, None)])
def test_block_scaled_fp16(oracle, capi, fmt, M, N, K, bias_dtype):
    import fp8linear_b200 as f

    x, w, b = _case(M, N, K, seed=M + N + K, bias_dtype=bias_dtype)
    if fmt == "mx":
        wq, ws = f.quantize_weight_mxfp8(w)
        out = f.mxfp8_linear(x, wq, ws, b)
        xq, xs = f.quantize_mxfp8(x)
        c = capi.mxfp8_gemm(xq, xs, wq, ws, b, out_dtype=torch.float16)
        ref = oracle.np_mxfp8_gemm(codes(xq), xs.cpu().numpy(), codes(wq), ws.cpu().numpy())
    else:
        wq, ws = f.quantize_weight_nvfp4(w)
        out = f.nvfp4_linear(x, wq, ws, b)
        xq, xs = f.quantize_nvfp4(x)
        c = capi.nvfp4_gemm(xq, xs, wq, ws, b, out_dtype=torch.float16)
        ref = oracle.np_nvfp4_gemm(xq.cpu().numpy(), xs.cpu().numpy(), wq.cpu().numpy(),
                                   ws.cpu().numpy())
    torch.cuda.synchronize()
    if b is not None:
        ref = ref + f32(b)[None, :]
    assert out.dtype == torch.float16 and out.shape == (M, N)
    assert torch.equal(out, c)
    assert max_rel(out.cpu(), torch.from_numpy(np.asarray(ref, np.float32))) <= OUT_TOL
