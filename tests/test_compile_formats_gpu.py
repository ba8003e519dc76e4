"""torch.compile (fullgraph, aot_eager) through the MXFP8, NVFP4 and modulated ops: their
fake implementations give the shapes and dtypes the trace needs, and the compiled function
returns the eager results."""
from __future__ import annotations

import pytest
import torch

from tests.helpers import require_sm100

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _dev():
    require_sm100()
    import fp8linear_b200  # noqa: F401


def test_compile_block_scaled_and_modulated_ops():
    import fp8linear_b200 as f

    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(2, 64, 256, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(320, 256, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(320, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    shift = (torch.randn(2, 256, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    scale = (torch.randn(2, 256, device="cuda", generator=g) * 0.2).to(torch.bfloat16)
    mq, ms = f.quantize_weight_mxfp8(w)
    nq, ns = f.quantize_weight_nvfp4(w)
    wq, ws = f.quantize_weight(w)

    def fn(x):
        a = f.mxfp8_linear(x, mq, ms, b)
        c = f.nvfp4_linear(x, nq, ns, b)
        d = f.fp8_linear_modulated(x, shift, scale, wq, ws, b)
        q, s = f.layernorm_modulate_quantize_fp8(x, shift, scale)
        e = f.fp8_linear(x, nq, ns, b)  # dispatch on the packed weight
        return a * 2.0, c + 1.0, d, q.view(torch.uint8), s, e

    eager = fn(x)
    out = torch.compile(fn, fullgraph=True, backend="aot_eager")(x)
    for o, r in zip(out, eager):
        assert o.dtype == r.dtype and o.shape == r.shape
        assert torch.equal(o, r)
