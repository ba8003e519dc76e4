"""The quantizer fused into the op before the linear (LayerNorm + AdaLN modulation +
per-token e4m3 quantization): the C oracle, its numpy twin and the unfused composition
in torch on the CPU (fp32 LayerNorm rounded to bf16, then the bf16 modulation ops, then the
reference's quantize rule)."""
from __future__ import annotations

import numpy as np
import pytest
import torch


def _case(M, K, B, dtype, seed, spread=3.0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g) * spread + 0.5
    shift = torch.randn(B, K, generator=g) * 0.1
    scale = torch.randn(B, K, generator=g) * 0.2
    return x.to(dtype), shift.to(dtype), scale.to(dtype)


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _torch_composition(x, shift, scale, eps=1e-6):
    M, K = x.shape
    b = torch.arange(M) // (M // shift.shape[0])
    ln = torch.nn.functional.layer_norm(x.float(), (K,), eps=eps).to(x.dtype)
    return ln * (1 + scale)[b] + shift[b]


@pytest.mark.parametrize("M,K,B,dtype", [(12, 96, 3, torch.bfloat16), (8, 3072, 2, torch.bfloat16),
                                         (10, 1032, 5, torch.float16), (4, 8192, 1, torch.bfloat16),
                                         (33, 264, 1, torch.float16)])
def test_oracle_c_and_numpy_agree(oracle, M, K, B, dtype):
    x, sh, sc = _case(M, K, B, dtype, seed=M * K)
    dt = oracle.BF16 if dtype == torch.bfloat16 else oracle.F16
    y, q, s = oracle.c_ln_modulate_quantize(_bits(x), _bits(sh), _bits(sc), 1e-6, dt)
    y2, q2, s2 = oracle.np_ln_modulate_quantize(_bits(x), _bits(sh), _bits(sc), 1e-6, dt)
    assert np.array_equal(y, y2) and np.array_equal(q, q2) and np.array_equal(s, s2)
    # the quantization step is exactly quantize_fp8's rule applied to y
    q3, s3 = oracle.c_quantize_rows(y, dt)
    assert np.array_equal(q, q3) and np.array_equal(s, s3)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_oracle_matches_unfused_torch(oracle, dtype):
    """The fixed-order fp32 statistics and IEEE rstd land on the same rounded values as
    torch's LayerNorm in nearly every element; where they differ it is by one unit of the
    last place of x's type."""
    x, sh, sc = _case(64, 3072, 2, dtype, seed=7)
    dt = oracle.BF16 if dtype == torch.bfloat16 else oracle.F16
    y, q, s = oracle.c_ln_modulate_quantize(_bits(x), _bits(sh), _bits(sc), 1e-6, dt)
    yt = _torch_composition(x, sh, sc)
    same = y == _bits(yt)
    assert same.mean() >= 0.999
    ours = torch.from_numpy(y.view(np.int16)).view(dtype).float()
    diff = (ours - yt.float()).abs()
    ulp = torch.finfo(dtype).eps * yt.float().abs().clamp_min(torch.finfo(dtype).tiny)
    assert bool((diff <= 1.01 * ulp).all())
    qt, st = oracle.c_quantize_rows(_bits(yt), dt)
    assert np.abs(s / st - 1).max() <= 2 ** -7


def test_oracle_edge_rows(oracle):
    """Constant rows (variance 0: rstd = 1/sqrt(eps)), a row with inf and NaN, tiny and
    huge magnitudes, fp16 overflow after modulation."""
    K = 256
    x = torch.zeros(6, K)
    x[0] = 3.0                                   # constant
    x[1, ::2] = float("inf"); x[1, 1::2] = 1.0    # inf
    x[2, 5] = float("nan")                        # NaN
    x[3] = torch.linspace(-1e-30, 1e-30, K)       # tiny
    x[4] = torch.linspace(-3e38, 3e38, K)         # huge (variance overflows)
    x[5] = torch.randn(K)
    sh = torch.full((2, K), 0.25)
    sc = torch.full((2, K), 50000.0)             # fp16: 1 + scale and products overflow
    for dtype, dt in ((torch.bfloat16, oracle.BF16), (torch.float16, oracle.F16)):
        xx = x.clamp(-60000, 60000) if dtype == torch.float16 else x
        xx = xx.clone(); xx[1, ::2] = float("inf"); xx[2, 5] = float("nan")
        y, q, s = oracle.c_ln_modulate_quantize(_bits(xx.to(dtype)), _bits(sh.to(dtype)),
                                               _bits(sc.to(dtype)), 1e-6, dt)
        y2, q2, s2 = oracle.np_ln_modulate_quantize(_bits(xx.to(dtype)), _bits(sh.to(dtype)),
                                                   _bits(sc.to(dtype)), 1e-6, dt)
        assert np.array_equal(q, q2) and np.array_equal(s, s2)
        # NaN-free rows of y agree bit for bit too
        ok = ~np.isnan(torch.from_numpy(y.view(np.int16)).view(dtype).float().numpy()).any(1)
        assert np.array_equal(y[ok], y2[ok])
        # quantize_fp8's rule on y: an inf in y (fp16 row 5 overflows after the
        # modulation) gives an inf scale, all-NaN-free rows a scale >= 1e-12
        assert (s >= 1e-12).all()
        if dtype == torch.float16:
            assert np.isinf(s[5])
