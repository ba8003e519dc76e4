"""fp8_linear with x and out in host memory (fp8lin_fp8_linear_host): row chunks whose
upload, kernels and download overlap on three streams must give the bits of the device
path, for several chunk counts (one chunk, a ragged last chunk of 488, 188 or 92 rows,
the few-token kernel for a single short chunk), dtypes, pageable buffers and calls back
to back. A ragged last chunk of a multi-chunk call runs the CTA-pair kernel like the
whole-M call, so even a tail short enough for the few-token kernel keeps the bits."""
from __future__ import annotations

import pytest
import torch

from fp8linear_b200.workloads import WORKLOADS, make_weight, make_x
from tests.helpers import require_sm100

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _dev():
    require_sm100()
    import fp8linear_b200  # noqa: F401


def _weights(N, K, seed=0, dtype=torch.bfloat16):
    import fp8linear_b200 as f

    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(dtype)
    b = (torch.randn(N, device="cuda", generator=g) * 0.02).to(dtype)
    wq, ws = f.quantize_weight(w)
    return wq, ws, b


@pytest.mark.parametrize("M,N,K,dtype", [(4608, 1024, 3072, torch.bfloat16),
                                         (1000, 776, 512, torch.float16),
                                         (100, 256, 256, torch.bfloat16),
                                         (700, 1024, 512, torch.bfloat16),
                                         (4700, 512, 1024, torch.bfloat16),
                                         (1, 264, 96, torch.bfloat16)])
def test_host_linear_matches_device(capi, M, N, K, dtype):
    wq, ws, b = _weights(N, K, seed=M, dtype=dtype)
    g = torch.Generator(device="cuda").manual_seed(M + 1)
    x = torch.randn(M, K, device="cuda", generator=g).to(dtype)
    want = capi.fp8_linear(x, wq, ws, b)
    out = capi.fp8_linear_host(x.cpu().pin_memory(), wq, ws, b)
    torch.cuda.current_stream().synchronize()
    assert out.dtype == dtype and out.shape == (M, N)
    assert torch.equal(out, want.cpu())


def test_host_linear_variants(capi):
    """No bias, fp16 out from bf16 x, pageable host buffers, two calls back to back on the
    library's streams (the second must not read the first one's chunks)."""
    import fp8linear_b200 as f

    wl = WORKLOADS["flux_qkv"]
    x = make_x(wl, gen_device="cuda")
    w, b = make_weight(wl, gen_device="cuda")
    wq, ws = f.quantize_weight(w)
    want = capi.fp8_linear(x, wq, ws, None, out=torch.empty(wl.M, wl.N, dtype=torch.float16,
                                                             device="cuda"))
    out = capi.fp8_linear_host(x.cpu(), wq, ws, None, out_host=torch.empty(wl.M, wl.N,
                                                                           dtype=torch.float16))
    x2 = make_x(wl, seed=5, gen_device="cuda")
    want2 = capi.fp8_linear(x2, wq, ws, b)
    out2 = capi.fp8_linear_host(x2.cpu().pin_memory(), wq, ws, b)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(out, want.cpu())
    assert torch.equal(out2, want2.cpu())


def test_host_linear_workspace_checked(capi):
    wq, ws, b = _weights(256, 256)
    x = torch.randn(600, 256, dtype=torch.bfloat16).pin_memory()
    small = torch.empty(1024, dtype=torch.uint8, device="cuda")
    with pytest.raises(RuntimeError, match="workspace"):
        capi.fp8_linear_host(x, wq, ws, b, workspace=small)


def test_host_linear_concurrent_callers(capi):
    """Several host threads calling at once on one device (ctypes drops the GIL): each
    call keeps its own chunks apart from the others' on the shared streams."""
    import threading

    wq, ws, b = _weights(512, 1024, seed=9)
    xs = [torch.randn(1500, 1024, dtype=torch.bfloat16).pin_memory() for _ in range(4)]
    want = [capi.fp8_linear(x.cuda(), wq, ws, b).cpu() for x in xs]
    outs = [None] * len(xs)

    def run(i):
        outs[i] = capi.fp8_linear_host(xs[i], wq, ws, b)
        torch.cuda.current_stream().synchronize()

    for _ in range(3):
        ts = [threading.Thread(target=run, args=(i,)) for i in range(len(xs))]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        for i in range(len(xs)):
            assert torch.equal(outs[i], want[i]), i
