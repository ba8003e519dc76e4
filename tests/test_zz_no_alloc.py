"""fp8lin_fp8_linear_noalloc through the C ABI, on the GPU.

This entry point is for callers that cannot allocate device memory (a plugin or
custom-op host that passes the op only its inputs and outputs and owns every other
byte of device memory, or a path that cannot take cudaMalloc's implicit device
synchronisation). It runs the same fused FP8 linear in a fixed 64 MiB scratch array
inside the library instead of a caller-provided workspace, so its outputs must match
fp8lin_fp8_linear's. Two calls in a row check that the scratch left by the first call
does not leak into the second. The file is named to be collected last.
"""
from __future__ import annotations

import pytest
import torch

from tests.helpers import OUT_TOL, max_rel, require_sm100

pytestmark = pytest.mark.gpu


def _case(M, K, N, seed):
    import fp8linear_b200 as f

    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(M, K, generator=g).bfloat16().cuda()
    w = (torch.randn(N, K, generator=g) * 0.02).bfloat16().cuda()
    b = (torch.randn(N, generator=g) * 0.02).bfloat16().cuda()
    wq, ws = f.quantize_weight(w)
    return x, wq, ws, b


def test_noalloc_matches_workspace_entry_point():
    require_sm100()
    from fp8linear_b200.capi import CApi

    api = CApi()
    cases = [_case(4608, 3072, 9216, seed=1), _case(333, 1024, 520, seed=2)]
    for x, wq, ws, b in cases:  # two calls in a row, different shapes and data
        got = api.fp8_linear_noalloc(x, wq, ws, b)
        ref = api.fp8_linear(x, wq, ws, b)
        torch.cuda.synchronize()
        assert max_rel(got, ref) <= OUT_TOL
        assert torch.equal(got, ref)  # same kernels on the same inputs: same bits
    assert api.device_status() == 0


def test_noalloc_rejects_sizes_beyond_scratch():
    require_sm100()
    from fp8linear_b200.capi import CApi, NOALLOC_SCRATCH_BYTES

    api = CApi()
    M, K = 8192, 8192  # 64 MiB of codes + 32 KiB of scales: one row too many
    assert api.workspace_size(M, K) > NOALLOC_SCRATCH_BYTES
    x = torch.empty(M, K, dtype=torch.bfloat16, device="cuda")
    wq = torch.empty(16, K, dtype=torch.float8_e4m3fn, device="cuda")
    ws = torch.ones(16, device="cuda")
    with pytest.raises(RuntimeError, match="scratch"):
        api.fp8_linear_noalloc(x, wq, ws)
