"""The CPU oracle itself: its e4m3 codec against torch's RNE cast, the scalar C
restatement against its vectorised numpy twin, and textbook known answers."""
from __future__ import annotations

import numpy as np
import pytest
import torch


def test_e4m3_codec_vs_torch(oracle):
    rng = np.random.default_rng(0)
    v = np.concatenate([rng.standard_normal(50_000).astype(np.float32) * s
                        for s in (1e-3, 0.05, 1, 30, 400)] +
                       [np.linspace(-448, 448, 20_001, dtype=np.float32)])
    lut = oracle.e4m3_decode_lut()
    fin = lut[np.isfinite(lut)]
    mids = ((fin[:-1] + fin[1:]) / 2).astype(np.float32)
    v = np.concatenate([v, mids, np.nextafter(mids, np.float32(1e9)),
                        np.nextafter(mids, np.float32(-1e9))])
    t = torch.from_numpy(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    # torch's cast does not saturate: it matches the non-saturating mode everywhere and
    # the saturating mode (the hardware convert) wherever |v| <= 448
    assert np.array_equal(oracle.np_e4m3_encode(v, saturate=False), t)
    inr = np.abs(v) <= 448
    assert np.array_equal(oracle.np_e4m3_encode(v[inr], saturate=True), t[inr])
    assert (oracle.np_e4m3_encode(v[~inr], saturate=True) & 0x7F == 0x7E).all()
    sample = v[inr][::97]
    c = np.array([oracle.c_e4m3_encode(s) for s in sample], np.uint8)
    assert np.array_equal(c, t[inr][::97])
    tl = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(lut, tl, equal_nan=True)


def test_e4m3_known_answers(oracle):
    kat = [(0.0, 0x00), (-0.0, 0x80), (1.0, 0x38), (1.0625, 0x38), (1.1875, 0x3A),
           (448.0, 0x7E), (-448.0, 0xFE), (2.0 ** -9, 0x01), (2.0 ** -10, 0x00),
           (3 * 2.0 ** -10, 0x02), (2.0 ** -6, 0x08), (500.0, 0x7E), (0.001953125 * 7, 0x07),
           (240.0, 0x77)]
    for v, code in kat:
        assert oracle.c_e4m3_encode(v, True) == code, v
    assert oracle.c_e4m3_encode(float("nan"), True) == 0x7F
    assert oracle.c_e4m3_encode(500.0, False) == 0x7F      # non-saturating cast -> NaN
    assert oracle.c_e4m3_encode(-500.0, False) == 0xFF


def _rand_bits(M, K, seed, dtype=np.float32, scale=1.0):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((M, K)) * scale).astype(np.float32)
    return torch.from_numpy(x)


@pytest.mark.parametrize("dt,code", [(torch.bfloat16, 0), (torch.float16, 1)])
def test_quantize_rows_c_vs_numpy(oracle, dt, code):
    x = _rand_bits(64, 1000, 1) * torch.logspace(-4, 3, 64)[:, None]
    x[3] = 0
    x[5, 7] = float("nan")
    x[6, 1] = float("inf")
    x[7, 2] = -float("inf")
    x16 = x.to(dt).view(torch.int16).numpy().view(np.uint16)
    cq, cs = oracle.c_quantize_rows(x16, code)
    nq, ns = oracle.np_quantize_rows(x16, code)
    assert np.array_equal(cq, nq)
    assert np.array_equal(cs.view(np.uint32), ns.view(np.uint32))
    assert cs[3] == np.float32(1e-12)


def test_quantize_rows_edge_semantics(oracle):
    """NaN inputs are ignored by the amax and clamp to -448; inf amax gives inv = 0."""
    row = np.array([np.nan, 1.0, -2.0, 448.0], np.float32)
    x16 = oracle.f32_to_bf16_bits(row[None, :])
    q, s = oracle.c_quantize_rows(x16, 0)
    assert s[0] == np.float32(1.0)
    assert list(q[0]) == [0xFE, 0x38, 0xC0, 0x7E]
    row = np.array([np.inf, 1.0, -3.0, 0.0], np.float32)
    q, s = oracle.c_quantize_rows(oracle.f32_to_bf16_bits(row[None, :]), 0)
    assert np.isinf(s[0])
    assert list(q[0]) == [0xFE, 0x00, 0x80, 0x00]   # inf*0=NaN->-448; finite*0 -> +-0


@pytest.mark.parametrize("recip", [True, False])
@pytest.mark.parametrize("dt,code", [(torch.bfloat16, 0), (torch.float16, 1), (torch.float32, 2)])
def test_quantize_weight_c_vs_numpy(oracle, recip, dt, code):
    w = _rand_bits(48, 520, 2, scale=0.02) * torch.logspace(-3, 2, 48)[:, None]
    w[0] = 0
    w = w.to(dt)
    arr = w.numpy() if dt == torch.float32 else w.view(torch.int16).numpy().view(np.uint16)
    cq, cs = oracle.c_quantize_weight(arr, code, recip)
    nq, ns = oracle.np_quantize_weight(arr, code, recip)
    assert np.array_equal(cq, nq)
    assert np.array_equal(cs.view(np.uint32), ns.view(np.uint32))


def test_weight_scale_reciprocal_vs_divide_differ_somewhere(oracle):
    """ATen's CUDA scalar divide (x * fl(1/448)) and a true divide disagree on some
    amax values; the oracle models the former (the reference's device)."""
    a = np.linspace(1e-3, 5.0, 200_001, dtype=np.float32)
    recip = (a * (np.float32(1.0) / np.float32(448.0))).astype(np.float32)
    div = (a / np.float32(448.0)).astype(np.float32)
    assert (recip != div).any()


def test_gemm_c_vs_port(oracle):
    rng = np.random.default_rng(3)
    M, N, K = 33, 40, 96
    xq, xs = oracle.np_quantize_rows(oracle.f32_to_bf16_bits(rng.standard_normal((M, K)).astype(np.float32)))
    wq, ws = oracle.np_quantize_weight(oracle.f32_to_bf16_bits((rng.standard_normal((N, K)) * 0.02).astype(np.float32)))
    b16 = (rng.standard_normal(N) * 0.02).astype(np.float16).view(np.uint16)
    c = oracle.c_gemm_dequant(xq, xs, wq, ws, b16, round_out=True)
    p = oracle.port_gemm_dequant(xq, xs, wq, ws, b16, round_out=True)
    assert np.array_equal(c.view(np.uint32), p.view(np.uint32))


def test_gemm_oracle_known_answer(oracle):
    """1x1 output: codes 1.0 * 2.0 over K=16, scales 0.5 and 3 -> 16*2*0.5*3 + bias."""
    xq = np.full((1, 16), 0x38, np.uint8)     # 1.0
    wq = np.full((1, 16), 0x40, np.uint8)     # 2.0
    out = oracle.c_gemm_dequant(xq, np.array([0.5], np.float32), wq, np.array([3.0], np.float32),
                                np.array([np.float16(0.25)]).view(np.uint16), round_out=False)
    assert out[0, 0] == np.float32(48.25)


@pytest.mark.parametrize("dt,code", [(torch.bfloat16, 0), (torch.float16, 1)])
def test_quantize_rows_torch_twin_vs_numpy(oracle, dt, code):
    """The multi-threaded torch twin (the timed CPU baseline's quantizer) gives the
    numpy twin's codes and scales bit for bit on finite rows: FLUX-like outliers, a zero
    row, values beyond 448 after scaling, tiny rows (subnormal codes), e4m3 midpoints."""
    g = torch.Generator().manual_seed(3)
    x = torch.randn(257, 1040, generator=g)
    x[:, ::97] *= 50
    x[3] = 0
    x[4, :5] = 448 * 3
    x[5] *= 1e-30 if dt == torch.bfloat16 else 1e-4
    lut = torch.from_numpy(oracle.e4m3_decode_lut())
    fin = lut[torch.isfinite(lut)].sort().values
    mids = (fin[:-1] + fin[1:]) / 2
    x[6, :mids.numel()] = mids
    x[6, -1] = 448.0
    xx = x.to(dt)
    q, sc = oracle.torch_quantize_rows(xx)
    nq, nsc = oracle.np_quantize_rows(xx.view(torch.int16).numpy().view(np.uint16), code)
    assert np.array_equal(q.view(torch.uint8).numpy(), nq)
    assert np.array_equal(sc.numpy().view(np.uint32), nsc.view(np.uint32))
