"""The NVFP4 oracle pinned to the reference: tests/golden/reference_nv_vectors.npz holds
outputs of the reference's own quantize_nvfp4 (compiled from its sources for sm_100a and
run on a B200 by tests/golden/make_golden_nv.py). The CPU restatement must reproduce its
packed e2m1 codes and tiled e4m3 scale grid bit for bit, for a block of every positive
finite bf16 and fp16 amax, edge rows and FLUX rows. The reference's nvfp4_gemm raises on
B200 (the file records its error), so the GEMM oracle is checked for its own consistency:
C against numpy, and against the per-block definition on a small case."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_nv_vectors.npz"
pytestmark = pytest.mark.skipif(not GOLDEN.exists(), reason="NVFP4 golden vectors not generated")


@pytest.fixture(scope="module")
def g():
    return dict(np.load(GOLDEN))


def _x(g, name):
    if f"{name}_x" in g:
        return g[f"{name}_x"]
    sys.path.insert(0, str(GOLDEN.parent))
    import make_golden_nv as G

    t = G.sweep_rows(torch.bfloat16 if name == "sweep" else torch.float16)
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("name", ["sweep", "sweep16", "edge", "edge16", "rows"])
def test_nv_quantize_matches_reference(g, oracle, name):
    x, dt, st = _x(g, name), int(g[f"{name}_dtype"]), int(g[f"{name}_code_stride"])
    cq, cs = oracle.c_quantize_nvfp4(x, dt)
    nq, ns = oracle.np_quantize_nvfp4(x, dt)
    assert np.array_equal(cs, g[f"{name}_scales"])
    assert np.array_equal(ns, g[f"{name}_scales"])
    assert np.array_equal(cq[::st], g[f"{name}_codes"])
    assert np.array_equal(cq, nq)


def test_nv_e2m1_thresholds(oracle):
    v = np.array([0.0, 0.2499, 0.25, 0.7499, 0.75, 1.25, 1.75, 2.5, 3.5, 4.99, 5.0, 6.0,
                  -0.25, -0.0, -0.1], np.float32)
    want = [0, 0, 1, 1, 2, 3, 4, 5, 6, 6, 7, 7, 9, 0, 8]
    assert list(oracle.np_e2m1_encode(v)) == want


def test_nv_gemm_oracle_consistent(oracle):
    rng = np.random.default_rng(3)
    x = torch.from_numpy(rng.standard_normal((20, 96)).astype(np.float32)).to(torch.bfloat16)
    w = torch.from_numpy((rng.standard_normal((24, 96)) * 0.02).astype(np.float32)).to(torch.bfloat16)
    xb = x.view(torch.int16).numpy().view(np.uint16)
    wb = w.view(torch.int16).numpy().view(np.uint16)
    xq, xs = oracle.c_quantize_nvfp4(xb)
    wq, ws = oracle.c_quantize_nvfp4(wb)
    c = oracle.c_nvfp4_gemm(xq, xs, wq, ws, round_out=False)
    n = oracle.np_nvfp4_gemm(xq, xs, wq, ws)
    assert oracle.max_rel_err(n, c) <= 1e-6
    # the definition, element by element, for one output
    a = oracle.np_nv_decode(xq, xs)[3]
    b = oracle.np_nv_decode(wq, ws)[5]
    assert abs(float(np.dot(a, b)) - float(c[3, 5])) <= 1e-6 * max(1.0, abs(float(c[3, 5])))
    assert "error" in str(np.load(GOLDEN)["gemm_error"]).lower()
