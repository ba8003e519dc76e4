"""The oracle pinned to the reference itself: tests/golden/reference_vectors.npz holds
outputs of the reference's own CUDA ops (compiled from its sources for sm_100a and
run on a B200 by tests/golden/make_golden.py). The CPU oracle must reproduce its e4m3
codes and scales bit for bit and its fp16 GEMM outputs within tolerance."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_vectors.npz"
pytestmark = pytest.mark.skipif(not GOLDEN.exists(), reason="golden vectors not generated")


@pytest.fixture(scope="module")
def g():
    return dict(np.load(GOLDEN))


@pytest.mark.parametrize("name,code", [("bf16", 0), ("f16", 1)])
def test_oracle_quantize_matches_reference(g, oracle, name, code):
    xq, xs = oracle.c_quantize_rows(g[f"x_{name}"], code)
    assert np.array_equal(xq, g[f"xq_{name}"])
    assert np.array_equal(xs.view(np.uint32), g[f"xs_{name}"].view(np.uint32))
    nq, ns = oracle.np_quantize_rows(g[f"x_{name}"], code)
    assert np.array_equal(nq, g[f"xq_{name}"])


def test_oracle_weight_quant_matches_reference(g, oracle):
    wq, ws = oracle.c_quantize_weight(g["w_bf16"], oracle.BF16, recip_scalar=True)
    assert np.array_equal(wq, g["wq"])
    assert np.array_equal(ws.view(np.uint32), g["ws"].view(np.uint32))


def test_oracle_weight_scale_is_reciprocal_multiply(g, oracle):
    """On these vectors the true-divide variant must differ somewhere from the
    reference's scales, or the vectors would not tell the two models apart."""
    _, ws_div = oracle.c_quantize_weight(g["w_bf16"], oracle.BF16, recip_scalar=False)
    _, ws_rec = oracle.c_quantize_weight(g["w_bf16"], oracle.BF16, recip_scalar=True)
    if np.array_equal(ws_div.view(np.uint32), ws_rec.view(np.uint32)):
        pytest.skip("vectors do not separate divide from reciprocal-multiply")
    assert not np.array_equal(ws_div.view(np.uint32), g["ws"].view(np.uint32))


def test_oracle_gemm_matches_reference(g, oracle):
    n = int(g["gemm_rows"])
    xq, xs = g["xq_bf16"][:n], g["xs_bf16"][:n]
    b = oracle.bf16_bits_to_f32(g["bias_bf16"])
    b16 = b.astype(np.float16).view(np.uint16)      # the reference rounds bias to fp16
    out = oracle.c_gemm_dequant(xq, xs, g["wq"], g["ws"], b16, round_out=True)
    ref = g["gemm_out_f16"].view(np.float16).astype(np.float32)
    # outputs past fp16's range overflow to +-inf in the reference's fp16 store; the
    # oracle's fp16 rounding must do the same
    fin = np.isfinite(ref)
    assert np.array_equal(np.isfinite(out), fin)
    assert np.array_equal(out[~fin], ref[~fin])
    assert oracle.max_rel_err(out[fin], ref[fin]) <= 1e-2
    # fp32 accumulation order is the only possible difference: almost all are identical
    assert np.mean(out == ref) > 0.9
