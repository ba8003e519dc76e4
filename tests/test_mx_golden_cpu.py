"""The MXFP8 oracle pinned to the reference: tests/golden/reference_mx_vectors.npz holds
outputs of the reference's own quantize_mxfp8 and mxfp8_gemm (compiled from its sources
for sm_100a and run on a B200 by tests/golden/make_golden_mx.py). The CPU restatement
must reproduce the e4m3 codes and the tiled e8m0 scale grid bit for bit, for every
positive finite bf16 and fp16 block amax, and the GEMM's fp16 outputs."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_mx_vectors.npz"
pytestmark = pytest.mark.skipif(not GOLDEN.exists(), reason="MX golden vectors not generated")


@pytest.fixture(scope="module")
def g():
    return dict(np.load(GOLDEN))


@pytest.mark.parametrize("name", ["sweep", "sweep16", "edge", "edge16", "rows"])
def test_mx_quantize_matches_reference(g, oracle, name):
    x, dt = g[f"{name}_x"], int(g[f"{name}_dtype"])
    cq, cs = oracle.c_quantize_mxfp8(x, dt)
    nq, ns = oracle.np_quantize_mxfp8(x, dt)
    assert np.array_equal(cs, g[f"{name}_scales"])
    assert np.array_equal(ns, g[f"{name}_scales"])
    assert np.array_equal(cq, nq)
    if f"{name}_codes" in g:
        assert np.array_equal(cq, g[f"{name}_codes"])


def test_mx_scale_grid_padding(g, oracle):
    """K = 96 has three blocks per row and M = 14 rows: the fourth scale column of the
    tile and rows 14..127 are padding, which holds 127 (e8m0 1.0)."""
    x = g["edge_x"]
    _, sc = oracle.c_quantize_mxfp8(x, oracle.BF16)
    assert sc.size == 512
    r = np.arange(128)
    pad_col = oracle.mx_sf_offset(r, 3, 1)
    assert np.all(sc[pad_col] == 127)
    rows_pad = oracle.mx_sf_offset(np.arange(14, 128)[:, None], np.arange(3)[None, :], 1)
    assert np.all(sc[rows_pad] == 127)


def test_mx_block_exponent_rule(oracle):
    """The exponent rule at its edges: powers of two, just below them, subnormals, the
    clamps, zero, NaN and inf."""
    vals = np.array([1.0, 1.9999999, 2.0, 448.0, 512.0, 2.0 ** -133, 2.0 ** -140,
                     3.3e38, 0.0, np.nan, np.inf], np.float32)
    want = [119, 119, 120, 127, 128, 0, 0, 246, 127, 127, 254]
    assert list(oracle.np_mx_block_exponent(vals)) == want


def test_mx_gemm_matches_reference(g, oracle):
    xq, xs = g["rows_codes"], g["rows_scales"]
    wq, ws = g["gemm_wq"], g["gemm_ws"]
    b16 = np.array([oracle.lib().oracle_f32_to_f16(float(v))
                    for v in oracle.bf16_bits_to_f32(g["gemm_b"])], np.uint16)
    ref = g["gemm_out_f16"].view(np.float16).astype(np.float32)
    out = oracle.c_mxfp8_gemm(xq, xs, wq, ws, b16, round_out=True)
    assert oracle.max_rel_err(out, ref) <= 1e-3
    outn = oracle.np_mxfp8_gemm(xq, xs, wq, ws, b16, round_out=True)
    assert oracle.max_rel_err(outn, ref) <= 1e-3
