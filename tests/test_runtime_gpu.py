"""Runtime behaviour on the GPU: the bounded-wait watchdog, side streams, CUDA graph
capture and torch.compile over the registered ops."""
from __future__ import annotations

import time

import pytest
import torch

from fp8linear_b200.workloads import WORKLOADS, make_weight, make_x
from tests.helpers import OUT_TOL, max_rel, require_sm100, torch_gemm_ref

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _dev():
    require_sm100()
    import fp8linear_b200  # noqa: F401


def _layer_inputs(name="flux_qkv"):
    import fp8linear_b200 as f

    wl = WORKLOADS[name]
    x = make_x(wl, gen_device="cuda")
    w, b = make_weight(wl, gen_device="cuda")
    wq, ws = f.quantize_weight(w)
    return x, wq, ws, b


def test_watchdog_wait_runs_out_and_context_survives(capi):
    """A wait that nothing completes ends at its limit with status 32; the kernel returns,
    the context stays usable and the regular kernels' status bits stay clear."""
    import fp8linear_b200 as f

    capi.device_status(clear=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    status = capi.selftest_watchdog(50_000)
    dt = time.perf_counter() - t0
    assert status == 32
    assert dt >= 0.045, dt
    assert dt < 5.0, dt
    # the device still runs work correctly afterwards
    x, wq, ws, b = _layer_inputs("sweep_M128")
    out = f.fp8_linear(x, wq, ws, b)
    xq, xs = f.quantize_fp8(x)
    assert max_rel(out, torch_gemm_ref(xq, xs, wq, ws, b)) <= OUT_TOL
    torch.cuda.synchronize()
    assert capi.device_status() == 0


def test_watchdog_argument_checks(capi):
    for bad in (0, 2_000_000):
        with pytest.raises(RuntimeError, match="status 1"):
            capi.selftest_watchdog(bad)


@pytest.mark.parametrize("name", ["flux_qkv", "sweep_M16"])
def test_side_stream_matches_default_stream(name):
    """Kernels launch on torch's current stream: the same call on a side stream gives the
    same bits as on the default stream."""
    import fp8linear_b200 as f

    x, wq, ws, b = _layer_inputs(name)
    ref = f.fp8_linear(x, wq, ws, b)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        out = f.fp8_linear(x, wq, ws, b)
    torch.cuda.current_stream().wait_stream(s)
    assert torch.equal(out, ref)


@pytest.mark.parametrize("name", ["flux_qkv", "sweep_M16"])
def test_cuda_graph_capture_and_replay(name):
    """fp8_linear captures into a CUDA graph (no allocation or sync inside the ops) and
    each replay recomputes from the current input buffer."""
    import fp8linear_b200 as f

    x, wq, ws, b = _layer_inputs(name)
    static_x = x.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            f.fp8_linear(static_x, wq, ws, b)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        static_out = f.fp8_linear(static_x, wq, ws, b)
    for seed in (1, 2):
        gen = torch.Generator(device="cuda").manual_seed(seed)
        new_x = torch.randn(x.shape, generator=gen, device="cuda", dtype=x.dtype)
        static_x.copy_(new_x)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(static_out, f.fp8_linear(new_x, wq, ws, b))
    del g


def test_torch_compile_fullgraph():
    """The ops trace through torch.compile without graph breaks (fake impls give the
    output shapes and dtypes) and the compiled module gives the eager result."""
    import fp8linear_b200 as f

    x, wq, ws, b = _layer_inputs("sweep_M128")

    def fn(x):
        y = f.fp8_linear(x, wq, ws, b)
        return y * 2.0

    eager = fn(x)
    compiled = torch.compile(fn, fullgraph=True, backend="aot_eager")
    out = compiled(x)
    assert out.dtype == eager.dtype and out.shape == eager.shape
    assert torch.equal(out, eager)
