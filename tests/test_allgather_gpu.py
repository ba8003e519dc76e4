"""Fused column-parallel linear (fp8lin_fp8_linear_allgather) on one GPU: extra local
buffers stand in for the peers' output buffers, so the epilogue's peer-store path is
checked without a second GPU. Every copy of this rank's column block must hold the same
bits, and no column outside the block may change. Against the plain fused linear on the
shard the block is bit-exact when both run the CTA-pair kernel (M > 256); for M <= 256 the
plain linear may run the split-K few-token kernel, whose fp32 summation order differs, so
there the check is OUT_TOL. With a
single buffer (no peers) the epilogue's paired stores write a column block of a wider
row pitch (ldo > N)."""
from __future__ import annotations

import pytest
import torch

from fp8linear_b200.sharding import column_range
from tests.helpers import OUT_TOL, max_rel, require_sm100

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("single", [False, True])
@pytest.mark.parametrize("M,N_total,K,world,rank",
                         [(300, 1024, 512, 2, 1), (4608, 3072, 3072, 4, 2), (129, 768, 256, 3, 0),
                          (65, 64, 128, 8, 7)])
def test_allgather_epilogue_writes_every_copy(M, N_total, K, world, rank, single, capi):
    require_sm100()
    import fp8linear_b200 as f

    g = torch.Generator(device="cpu").manual_seed(M + N_total)
    x = torch.randn(M, K, generator=g).bfloat16().cuda()
    w = (torch.randn(N_total, K, generator=g) * 0.02).bfloat16().cuda()
    b = (torch.randn(N_total, generator=g) * 0.02).bfloat16().cuda()
    wq, ws = f.quantize_weight(w)
    s, e = column_range(N_total, world, rank)
    ref = f.fp8_linear(x, wq[s:e].contiguous(), ws[s:e].contiguous(), b[s:e].contiguous())
    n_copies = 1 if single else min(world, 3)
    sentinel = torch.tensor(-7.0, dtype=torch.bfloat16)
    bufs = [torch.full((M, N_total), float(sentinel), dtype=torch.bfloat16, device="cuda")
            for _ in range(n_copies)]
    ptrs = [t.data_ptr() + s * t.element_size() for t in bufs]
    capi.fp8_linear_allgather(x, wq[s:e].contiguous(), ws[s:e].contiguous(),
                              b[s:e].contiguous(), ptrs, ldo=N_total)
    torch.cuda.synchronize()
    first = bufs[0][:, s:e]
    if M > 256:
        assert torch.equal(first, ref)
    else:
        assert max_rel(first.float().cpu(), ref.float().cpu()) <= OUT_TOL
    for t in bufs:
        assert torch.equal(t[:, s:e], first)
        outside = torch.cat([t[:, :s].flatten(), t[:, e:].flatten()])
        assert (outside == sentinel).all()
    assert capi.device_status() == 0
