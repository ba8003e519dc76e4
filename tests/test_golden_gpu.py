"""Our kernels against the reference's own outputs stored in
tests/golden/reference_vectors.npz (see tests/golden/make_golden.py)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from tests.helpers import OUT_TOL, max_rel, require_sm100

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_vectors.npz"
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not GOLDEN.exists(), reason="golden vectors not generated")]


@pytest.fixture(scope="module")
def g():
    require_sm100()
    return dict(np.load(GOLDEN))


def _dev16(a: np.ndarray, dt) -> torch.Tensor:
    return torch.from_numpy(a.view(np.int16).copy()).view(dt).cuda()


@pytest.mark.parametrize("name,dt", [("bf16", torch.bfloat16), ("f16", torch.float16)])
def test_quantize_matches_reference_vectors(g, name, dt):
    import fp8linear_b200 as f

    xq, xs = f.quantize_fp8(_dev16(g[f"x_{name}"], dt))
    assert np.array_equal(xq.cpu().view(torch.uint8).numpy(), g[f"xq_{name}"])
    assert np.array_equal(xs.cpu().numpy().view(np.uint32), g[f"xs_{name}"].view(np.uint32))


def test_weight_and_gemm_match_reference_vectors(g):
    import fp8linear_b200 as f

    w = _dev16(g["w_bf16"], torch.bfloat16)
    wq, ws = f.quantize_weight(w)
    assert np.array_equal(wq.cpu().view(torch.uint8).numpy(), g["wq"])
    assert np.array_equal(ws.cpu().numpy().view(np.uint32), g["ws"].view(np.uint32))
    n = int(g["gemm_rows"])
    xq = torch.from_numpy(g["xq_bf16"][:n].copy()).cuda().view(torch.float8_e4m3fn)
    xs = torch.from_numpy(g["xs_bf16"][:n].copy()).cuda()
    b = _dev16(g["bias_bf16"], torch.bfloat16)
    out = f.fp8_gemm(xq, xs, wq, ws, b)
    ref = torch.from_numpy(g["gemm_out_f16"].view(np.float16).astype(np.float32))
    got = out.float().cpu()
    fin = torch.isfinite(ref)
    # where the reference's fp16 output overflowed, the bf16 output is beyond fp16 range
    assert (got[~fin].abs() > 65504).all() and torch.equal(got[~fin].sign(), ref[~fin].sign())
    assert max_rel(got[fin], ref[fin]) <= OUT_TOL
