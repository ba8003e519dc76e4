"""CPU oracle for the per-channel FP8 linear path of drbh/fp8linear.

TEST INFRASTRUCTURE ONLY: the oracle for fp8linear_b200's CUDA kernels. Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import it. The product package never imports anything under ``oracle/``.

Two restatements of the same algorithm live here:

* ``C`` -- ``fp8_oracle.c`` through ctypes: scalar, one element at a time, the
  primary restatement (see the citations in that file).
* ``np_*`` / ``port_*`` -- vectorised numpy/torch versions of the same steps, used
  at sizes where the scalar code would take too long and as the timed CPU
  baseline (the "torch emulation" CPU path: per-token e4m3 quant, fp32 matmul of
  the codes, dequant + bias). Tests check them against the C restatement.

Reference citations (paths relative to the reference project root):
  activation quant     csrc/quantize.cu:45-73 (kernel), :199-234 (host op)
  weight quant         csrc/quantize.cu:359-365
  GEMM + dequant/bias  csrc/fp8_gemm.cu:139-194, dequant_bias_kernel :65-80
  fused entry          csrc/fp8_gemm.cu:196-221
  MXFP8 block quant    csrc/quantize.cu:75-131 (layout + kernel), :239-285 (host op)
  MXFP8 GEMM           csrc/fp8_gemm.cu:233-333 (cuBLASLt VEC32_UE8M0, bias, fp16 out)
  NVFP4 quant          csrc/quantize.cu:136-194 (f2e2m1 + kernel), :290-334 (host op)
  NVFP4 GEMM           csrc/fp8_gemm.cu:347-446 (cuBLASLt VEC16_UE4M3, bias, fp16 out)
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "fp8_oracle.c"
BUILD_DIR = HERE / "_build"
LIB_PATH = BUILD_DIR / "liboracle.so"

E4M3_MAX = np.float32(448.0)
SCALE_FLOOR = np.float32(1e-12)
BF16, F16, F32 = 0, 1, 2


# ----------------------------------------------------------------------------- build


def build() -> Path:
    """Compile fp8_oracle.c into oracle/_build/liboracle.so (skipped when fresh)."""
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    if LIB_PATH.exists() and LIB_PATH.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(f".so.{os.getpid()}")
    cmd = ["cc", "-O2", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
           "-std=c11", str(SRC), "-o", str(tmp), "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = build()
        L = ctypes.CDLL(str(path))
        P = ctypes.c_void_p
        i64 = ctypes.c_int64
        L.oracle_e4m3_encode.argtypes = [ctypes.c_float, ctypes.c_int]
        L.oracle_e4m3_encode.restype = ctypes.c_uint8
        L.oracle_e4m3_decode.argtypes = [ctypes.c_uint8]
        L.oracle_e4m3_decode.restype = ctypes.c_float
        L.oracle_quantize_rows.argtypes = [P, ctypes.c_int, i64, i64, P, P]
        L.oracle_quantize_rows.restype = None
        L.oracle_quantize_weight.argtypes = [P, ctypes.c_int, i64, i64, ctypes.c_int, P, P]
        L.oracle_quantize_weight.restype = None
        L.oracle_gemm_dequant.argtypes = [P, P, P, P, P, i64, i64, i64, ctypes.c_int, P, P]
        L.oracle_gemm_dequant.restype = None
        L.oracle_f32_to_f16.argtypes = [ctypes.c_float]
        L.oracle_f32_to_f16.restype = ctypes.c_uint16
        L.oracle_mx_sf_bytes.argtypes = [i64, i64]
        L.oracle_mx_sf_bytes.restype = i64
        L.oracle_quantize_mxfp8.argtypes = [P, ctypes.c_int, i64, i64, P, P]
        L.oracle_quantize_mxfp8.restype = None
        L.oracle_mxfp8_gemm.argtypes = [P, P, P, P, P, i64, i64, i64, ctypes.c_int, P]
        L.oracle_mxfp8_gemm.restype = None
        L.oracle_quantize_nvfp4.argtypes = [P, ctypes.c_int, i64, i64, P, P]
        L.oracle_quantize_nvfp4.restype = None
        L.oracle_nvfp4_gemm.argtypes = [P, P, P, P, P, i64, i64, i64, ctypes.c_int, P]
        L.oracle_nvfp4_gemm.restype = None
        L.oracle_ln_modulate_quantize.argtypes = [P, ctypes.c_int, i64, i64, i64, P, P,
                                                  ctypes.c_float, P, P, P]
        L.oracle_ln_modulate_quantize.restype = None
        _lib = L
    return _lib


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ----------------------------------------------------------------------------- C restatement


def c_quantize_rows(x16: np.ndarray, dtype: int = BF16):
    """x16: uint16 [M, K] holding bf16 (dtype 0) or fp16 (dtype 1) bit patterns."""
    x16 = np.ascontiguousarray(x16, dtype=np.uint16)
    M, K = x16.shape
    xq = np.empty((M, K), np.uint8)
    sc = np.empty((M,), np.float32)
    lib().oracle_quantize_rows(_ptr(x16), dtype, M, K, _ptr(xq), _ptr(sc))
    return xq, sc


def c_quantize_weight(w: np.ndarray, dtype: int = BF16, recip_scalar: bool = True):
    """w: uint16 bit patterns (bf16/fp16) or float32 [N, K]."""
    w = np.ascontiguousarray(w)
    N, K = w.shape
    wq = np.empty((N, K), np.uint8)
    sc = np.empty((N,), np.float32)
    lib().oracle_quantize_weight(_ptr(w), dtype, N, K, int(recip_scalar), _ptr(wq), _ptr(sc))
    return wq, sc


def c_gemm_dequant(xq, xs, wq, ws, bias16=None, round_out=True, want_acc=False):
    xq = np.ascontiguousarray(xq, np.uint8)
    wq = np.ascontiguousarray(wq, np.uint8)
    xs = np.ascontiguousarray(xs, np.float32)
    ws = np.ascontiguousarray(ws, np.float32)
    if bias16 is not None:
        bias16 = np.ascontiguousarray(bias16, np.uint16)
    M, K = xq.shape
    N = wq.shape[0]
    out = np.empty((M, N), np.float32)
    acc = np.empty((M, N), np.float32) if want_acc else None
    lib().oracle_gemm_dequant(_ptr(xq), _ptr(xs), _ptr(wq), _ptr(ws), _ptr(bias16),
                              M, N, K, int(round_out), _ptr(acc), _ptr(out))
    return (out, acc) if want_acc else out


def mx_sf_bytes(rows: int, K: int) -> int:
    """Bytes of the padded MXFP8 scale grid: ceil(rows/128) * ceil((K/32)/4) * 512."""
    return ((rows + 127) // 128) * ((K // 32 + 3) // 4) * 512


def mx_sf_offset(r, c, ncb):
    """Offset of block scale (row r, block c) in the tiled layout (csrc/quantize.cu:80-83);
    works elementwise on numpy integer arrays."""
    return (r // 128) * (ncb * 512) + (c // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + (c % 4)


def c_quantize_mxfp8(x16: np.ndarray, dtype: int = BF16):
    """MXFP8 codes [M, K] and the tiled e8m0 scale grid (1-D uint8)."""
    x16 = np.ascontiguousarray(x16, dtype=np.uint16)
    M, K = x16.shape
    xq = np.empty((M, K), np.uint8)
    sc = np.empty((mx_sf_bytes(M, K),), np.uint8)
    lib().oracle_quantize_mxfp8(_ptr(x16), dtype, M, K, _ptr(xq), _ptr(sc))
    return xq, sc


def c_mxfp8_gemm(xq, xs, wq, ws, bias16=None, round_out=True):
    xq = np.ascontiguousarray(xq, np.uint8)
    wq = np.ascontiguousarray(wq, np.uint8)
    xs = np.ascontiguousarray(xs, np.uint8)
    ws = np.ascontiguousarray(ws, np.uint8)
    if bias16 is not None:
        bias16 = np.ascontiguousarray(bias16, np.uint16)
    M, K = xq.shape
    N = wq.shape[0]
    out = np.empty((M, N), np.float32)
    lib().oracle_mxfp8_gemm(_ptr(xq), _ptr(xs), _ptr(wq), _ptr(ws), _ptr(bias16), M, N, K,
                            int(round_out), _ptr(out))
    return out


def nv_sf_bytes(rows: int, K: int) -> int:
    """Bytes of the NVFP4 scale grid: ceil(rows/128) * ceil((K/16)/4) * 512."""
    return ((rows + 127) // 128) * ((K // 16 + 3) // 4) * 512


def c_quantize_nvfp4(x16: np.ndarray, dtype: int = BF16):
    """NVFP4 packed codes [M, K/2] and the tiled e4m3 scale grid (1-D uint8)."""
    x16 = np.ascontiguousarray(x16, dtype=np.uint16)
    M, K = x16.shape
    xq = np.empty((M, K // 2), np.uint8)
    sc = np.empty((nv_sf_bytes(M, K),), np.uint8)
    lib().oracle_quantize_nvfp4(_ptr(x16), dtype, M, K, _ptr(xq), _ptr(sc))
    return xq, sc


def c_nvfp4_gemm(xq, xs, wq, ws, bias16=None, round_out=True):
    xq = np.ascontiguousarray(xq, np.uint8)
    wq = np.ascontiguousarray(wq, np.uint8)
    xs = np.ascontiguousarray(xs, np.uint8)
    ws = np.ascontiguousarray(ws, np.uint8)
    if bias16 is not None:
        bias16 = np.ascontiguousarray(bias16, np.uint16)
    M, K = xq.shape[0], xq.shape[1] * 2
    N = wq.shape[0]
    out = np.empty((M, N), np.float32)
    lib().oracle_nvfp4_gemm(_ptr(xq), _ptr(xs), _ptr(wq), _ptr(ws), _ptr(bias16), M, N, K,
                            int(round_out), _ptr(out))
    return out


def c_ln_modulate_quantize(x16, shift16, scale16, eps=1e-6, dtype: int = BF16):
    """LayerNorm + AdaLN modulation + per-token quantization (oracle_ln_modulate_quantize).
    x16 uint16 [M, K]; shift16 / scale16 uint16 [B, K] (B divides M). Returns
    (y uint16 [M, K], xq uint8 [M, K], xs float32 [M])."""
    x16 = np.ascontiguousarray(x16, np.uint16)
    shift16 = np.ascontiguousarray(shift16, np.uint16)
    scale16 = np.ascontiguousarray(scale16, np.uint16)
    M, K = x16.shape
    y = np.empty((M, K), np.uint16)
    xq = np.empty((M, K), np.uint8)
    xs = np.empty((M,), np.float32)
    lib().oracle_ln_modulate_quantize(_ptr(x16), dtype, M, K, shift16.shape[0], _ptr(shift16),
                                      _ptr(scale16), float(eps), _ptr(y), _ptr(xq), _ptr(xs))
    return y, xq, xs


def c_e4m3_encode(v: float, saturate: bool = True) -> int:
    return int(lib().oracle_e4m3_encode(float(v), int(saturate)))


# ----------------------------------------------------------------------------- numpy port


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (h.astype(np.uint32) << 16).view(np.float32)


def f16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return h.view(np.float16).astype(np.float32)


def f32_to_bf16_bits(f: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (NaN kept quiet)."""
    u = np.ascontiguousarray(f, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r = np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)
    return r


def np_e4m3_encode(v: np.ndarray, saturate: bool = True) -> np.ndarray:
    """Vectorised twin of oracle_e4m3_encode (RNE, same saturate semantics)."""
    v = np.ascontiguousarray(v, np.float32)
    u = v.view(np.uint32)
    sign = ((u >> 24) & 0x80).astype(np.uint8)
    a_bits = u & np.uint32(0x7FFFFFFF)
    af = a_bits.view(np.float32)
    # normal path
    e = (a_bits >> 23).astype(np.int32) - 127
    m = a_bits & np.uint32(0x7FFFFF)
    keep = (m >> 20).astype(np.int32)
    rem = m & np.uint32(0xFFFFF)
    up = (rem > 0x80000) | ((rem == 0x80000) & ((keep & 1) == 1))
    keep = keep + up.astype(np.int32)
    carry = keep == 8
    keep = np.where(carry, 0, keep)
    e = e + carry.astype(np.int32)
    normal = (((e + 7) << 3) | keep).astype(np.int32)
    # subnormal path (below 2^-6)
    with np.errstate(invalid="ignore", over="ignore"):
        sub = np.rint(af * np.float32(512.0))
        sub = np.where(np.isfinite(sub), sub, 0).astype(np.int32)
    code = np.where(af < np.float32(0.015625), sub, normal)
    code = np.where(af > E4M3_MAX, 0x7E, code)
    big = af >= np.float32(464.0)
    nan = a_bits > 0x7F800000
    if saturate:
        code = np.where(big, 0x7E, code)
        res = (code.astype(np.uint8) | sign)
        res = np.where(nan, np.uint8(0x7F), res)
    else:
        code = np.where(big | nan, 0x7F, code)
        res = code.astype(np.uint8) | sign
    return res.astype(np.uint8)


_DECODE_LUT = None


def e4m3_decode_lut() -> np.ndarray:
    global _DECODE_LUT
    if _DECODE_LUT is None:
        b = np.arange(256, dtype=np.uint32)
        s = (b & 0x80) != 0
        e = (b >> 3) & 0xF
        m = b & 7
        sub = m.astype(np.float32) * np.float32(2.0 ** -9)
        nrm = ((e + 120) << 23 | (m << 20)).astype(np.uint32).view(np.float32)
        v = np.where(e == 0, sub, nrm).astype(np.float32)
        v = np.where((e == 15) & (m == 7), np.float32(np.nan), v)
        _DECODE_LUT = np.where(s, -v, v).astype(np.float32)
    return _DECODE_LUT


def np_quantize_rows(x16: np.ndarray, dtype: int = BF16):
    """Vectorised twin of oracle_quantize_rows (bit-identical)."""
    x16 = np.ascontiguousarray(x16, np.uint16)
    xf = bf16_bits_to_f32(x16) if dtype == BF16 else f16_bits_to_f32(x16)
    if xf.shape[0] == 0:
        return np.empty(xf.shape, np.uint8), np.empty((0,), np.float32)
    amax = np.fmax.reduce(np.abs(xf), axis=1, initial=np.float32(0.0)).astype(np.float32)
    sc = np.fmax(amax / E4M3_MAX, SCALE_FLOOR).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        inv = (np.float32(1.0) / sc).astype(np.float32)
        p = (xf * inv[:, None]).astype(np.float32)
    c = np.fmin(np.fmax(p, -E4M3_MAX), E4M3_MAX)
    return np_e4m3_encode(c, saturate=True), sc


def torch_quantize_rows(x):
    """Per-token quantization of a CPU tensor x [M, K] (bf16/fp16) with multi-threaded
    torch ops: the reference's rule (csrc/quantize.cu:52-72) as its torch emulation
    writes it. amax in fp32, sc = max(amax / 448, 1e-12), inv = 1 / sc (IEEE fp32
    divides), codes = e4m3(clamp(x * inv, -448, 448)) with torch's round-to-nearest-even
    cast. Bit-identical to np_quantize_rows on finite inputs (torch's amax propagates a
    NaN where the kernel's fmaxf ignores it). Returns (codes as torch.float8_e4m3fn,
    scales fp32)."""
    import torch

    xf = x.float()
    amax = xf.abs().amax(dim=1)
    lim = float(E4M3_MAX)
    sc = torch.clamp_min(amax / lim, float(SCALE_FLOOR))
    inv = 1.0 / sc
    q = xf.mul_(inv[:, None]).clamp_(-lim, lim).to(torch.float8_e4m3fn)
    return q, sc


def _np_round_to(f: np.ndarray, dtype: int) -> np.ndarray:
    f = np.ascontiguousarray(f, np.float32)
    if dtype == BF16:
        return bf16_bits_to_f32(f32_to_bf16_bits(f))
    return f.astype(np.float16).astype(np.float32)


def _np_lane_tree(part: np.ndarray) -> np.ndarray:
    idx = np.arange(32)
    for o in (16, 8, 4, 2, 1):
        part = (part + part[:, idx ^ o]).astype(np.float32)
    return part[:, 0]


def np_ln_modulate_quantize(x16, shift16, scale16, eps=1e-6, dtype: int = BF16):
    """Vectorised twin of oracle_ln_modulate_quantize (bit-identical)."""
    x16 = np.ascontiguousarray(x16, np.uint16)
    M, K = x16.shape
    B = shift16.shape[0]
    to32 = bf16_bits_to_f32 if dtype == BF16 else f16_bits_to_f32
    xf = to32(x16)
    nch = K // 8
    chunks = xf.reshape(M, nch, 8)
    kf = np.float32(K)

    def lane_sums(vals):  # vals [M, nch, 8] float32 -> lane partials [M, 32]
        part = np.zeros((M, 32), np.float32)
        for i in range(-(-nch // 32)):
            lo, hi = 32 * i, min(32 * i + 32, nch)
            for e in range(8):
                part[:, : hi - lo] = (part[:, : hi - lo] + vals[:, lo:hi, e]).astype(np.float32)
        return part

    with np.errstate(invalid="ignore", over="ignore"):
        mean = (_np_lane_tree(lane_sums(chunks)) / kf).astype(np.float32)
        d = (chunks - mean[:, None, None]).astype(np.float32)
        var = (_np_lane_tree(lane_sums((d * d).astype(np.float32))) / kf).astype(np.float32)
        rstd = (np.float32(1.0) / np.sqrt((var + np.float32(eps)).astype(np.float32))).astype(np.float32)
        b = np.arange(M) // (M // B)
        sc = to32(np.ascontiguousarray(scale16, np.uint16))[b]
        sh = to32(np.ascontiguousarray(shift16, np.uint16))[b]
        ln = _np_round_to(((xf - mean[:, None]).astype(np.float32) * rstd[:, None]).astype(np.float32), dtype)
        m1 = _np_round_to((np.float32(1.0) + sc).astype(np.float32), dtype)
        t = _np_round_to((ln * m1).astype(np.float32), dtype)
        y = _np_round_to((t + sh).astype(np.float32), dtype)
    y16 = f32_to_bf16_bits(y) if dtype == BF16 else y.astype(np.float16).view(np.uint16)
    xq, xs = np_quantize_rows(y16, dtype)
    return y16, xq, xs


def np_quantize_weight(w: np.ndarray, dtype: int = BF16, recip_scalar: bool = True):
    """Vectorised twin of oracle_quantize_weight (bit-identical, NaN sign aside)."""
    if dtype == F32:
        wf = np.ascontiguousarray(w, np.float32)
    else:
        w16 = np.ascontiguousarray(w, np.uint16)
        wf = bf16_bits_to_f32(w16) if dtype == BF16 else f16_bits_to_f32(w16)
    a = np.abs(wf)
    amax = np.max(a, axis=1, initial=np.float32(0.0)).astype(np.float32)  # NaN propagates
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        if recip_scalar:
            s = (amax * (np.float32(1.0) / E4M3_MAX)).astype(np.float32)
        else:
            s = (amax / E4M3_MAX).astype(np.float32)
        sc = np.where(np.isnan(s), s, np.maximum(s, SCALE_FLOOR)).astype(np.float32)
        q = (wf / sc[:, None]).astype(np.float32)
    c = np.where(np.isnan(q), q, np.clip(q, -E4M3_MAX, E4M3_MAX)).astype(np.float32)
    return np_e4m3_encode(c, saturate=False), sc


def port_gemm_dequant(xq, xs, wq, ws, bias16=None, round_out=True, acc_dtype="float64",
                      threads: int | None = None):
    """Vectorised twin of oracle_gemm_dequant; the matmul runs in torch on the CPU.

    acc_dtype "float64" gives the exact-sum reference (tests); "float32" is the
    reference's own fp32-accumulate arithmetic (the timed CPU baseline).
    """
    import torch

    if threads is not None:
        torch.set_num_threads(threads)
    lut = torch.from_numpy(e4m3_decode_lut())
    tdt = torch.float64 if acc_dtype == "float64" else torch.float32
    a = lut[torch.from_numpy(np.ascontiguousarray(xq, np.uint8)).long()].to(tdt)
    b = lut[torch.from_numpy(np.ascontiguousarray(wq, np.uint8)).long()].to(tdt)
    acc = (a @ b.T).to(torch.float32)
    t = acc * torch.from_numpy(np.ascontiguousarray(xs, np.float32))[:, None]
    v = t * torch.from_numpy(np.ascontiguousarray(ws, np.float32))[None, :]
    if bias16 is not None:
        bh = torch.from_numpy(np.ascontiguousarray(bias16, np.uint16).view(np.float16))
        v = v + bh.float()[None, :]
    if round_out:
        v = v.half().float()
    return v.numpy()


def port_linear(x16: np.ndarray, wq, ws, bias16=None, dtype: int = BF16, acc_dtype="float32",
                round_out=True):
    """Whole reference CPU path (fp8_linear, csrc/fp8_gemm.cu:196-221) on a 2-D x."""
    xq, xs = np_quantize_rows(x16, dtype)
    return port_gemm_dequant(xq, xs, wq, ws, bias16, round_out=round_out, acc_dtype=acc_dtype)


# ----------------------------------------------------------------------------- checks


def max_rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    """max|got - ref| / max|ref| in fp32 (the tolerance measure for outputs)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    denom = np.max(np.abs(ref)) if ref.size else 0.0
    if ref.size == 0:
        return 0.0
    return float(np.max(np.abs(got - ref)) / max(denom, 1e-30))


def norm_rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    """||got - ref|| / ||ref|| (the measure scripts/mxfp8_check.py:62 prints)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))


# ----------------------------------------------------------------------------- MXFP8 numpy twins


def np_mx_block_exponent(amax: np.ndarray) -> np.ndarray:
    """e8m0 block scale from block amax (float32 array), the rule of
    oracle_quantize_mxfp8: clamp(exponent(amax) - 8 + 127, 0, 254) for amax > 0
    (254 for inf), 127 for zero and NaN."""
    a = np.asarray(amax, np.float32)
    with np.errstate(invalid="ignore"):
        _, e2 = np.frexp(np.where(np.isfinite(a) & (a > 0), a, np.float32(1.0)))
    e8 = np.clip(e2.astype(np.int64) - 1 - 8 + 127, 0, 254)
    e8 = np.where(np.isinf(a), 254, e8)
    with np.errstate(invalid="ignore"):
        pos = a > 0
    return np.where(pos, e8, 127).astype(np.uint8)


def np_quantize_mxfp8(x16: np.ndarray, dtype: int = BF16):
    """Vectorised twin of c_quantize_mxfp8."""
    x16 = np.ascontiguousarray(x16, dtype=np.uint16)
    M, K = x16.shape
    nblk, ncb = K // 32, (K // 32 + 3) // 4
    x = bf16_bits_to_f32(x16) if dtype == BF16 else f16_bits_to_f32(x16)
    blk = np.abs(x.reshape(M, nblk, 32))
    all_nan = np.all(np.isnan(blk), axis=2)
    amax = np.max(np.where(np.isnan(blk), np.float32(-1.0), blk), axis=2)
    amax = np.where(all_nan, np.float32(np.nan), amax).astype(np.float32)
    e8 = np_mx_block_exponent(amax)
    inv = np.ldexp(np.float32(1.0), (127 - e8.astype(np.int32))).astype(np.float32)
    with np.errstate(invalid="ignore", over="ignore"):
        p = (x.reshape(M, nblk, 32) * inv[:, :, None]).astype(np.float32)
    c = np.minimum(np.maximum(p, -E4M3_MAX), E4M3_MAX)  # numpy max/min propagate NaN
    c = np.where(np.isnan(p), -E4M3_MAX, c)             # fminf(fmaxf(NaN, -448), 448) = -448
    xq = np_e4m3_encode(c.reshape(M, K), saturate=True)
    sc = np.full((mx_sf_bytes(M, K),), 127, np.uint8)
    r, g = np.meshgrid(np.arange(M), np.arange(nblk), indexing="ij")
    sc[mx_sf_offset(r, g, ncb)] = e8
    return xq, sc


def np_mx_decode(q: np.ndarray, sc: np.ndarray) -> np.ndarray:
    """float64 values of MXFP8 codes [R, K] with their tiled scale grid."""
    R, K = q.shape
    nblk, ncb = K // 32, (K // 32 + 3) // 4
    r, g = np.meshgrid(np.arange(R), np.arange(nblk), indexing="ij")
    e8 = sc[mx_sf_offset(r, g, ncb)].astype(np.int64)
    dec = e4m3_decode_lut().astype(np.float64)[q].reshape(R, nblk, 32)
    return (dec * np.ldexp(1.0, e8 - 127)[:, :, None]).reshape(R, K)


def np_mxfp8_gemm(xq, xs, wq, ws, bias16=None, round_out=False):
    """Decoded float64 matmul (twin of c_mxfp8_gemm up to summation order)."""
    acc = (np_mx_decode(xq, xs) @ np_mx_decode(wq, ws).T).astype(np.float32)
    if bias16 is not None:
        acc = acc + f16_bits_to_f32(np.asarray(bias16, np.uint16))[None, :]
    if round_out:
        acc = acc.astype(np.float16).astype(np.float32)
    return acc


# ----------------------------------------------------------------------------- NVFP4 numpy twins

E2M1_MAG = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], np.float32)


def np_e2m1_encode(v: np.ndarray) -> np.ndarray:
    """Vectorised oracle_e2m1_encode (threshold rounding, sign only for v < 0)."""
    v = np.asarray(v, np.float32)
    with np.errstate(invalid="ignore"):
        s = np.where(v < 0, 8, 0).astype(np.uint8)
    a = np.abs(v)
    c = np.searchsorted(np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32), a,
                        side="right").astype(np.uint8)
    c = np.where(np.isnan(a), 7, c)  # unreachable after the clamp; NaN sorts last
    return s | c


def np_quantize_nvfp4(x16: np.ndarray, dtype: int = BF16):
    """Vectorised twin of c_quantize_nvfp4."""
    x16 = np.ascontiguousarray(x16, dtype=np.uint16)
    M, K = x16.shape
    nblk, ncb = K // 16, (K // 16 + 3) // 4
    x = bf16_bits_to_f32(x16) if dtype == BF16 else f16_bits_to_f32(x16)
    blk = x.reshape(M, nblk, 16)
    a = np.abs(blk)
    all_nan = np.all(np.isnan(a), axis=2)
    amax = np.max(np.where(np.isnan(a), np.float32(-1.0), a), axis=2).astype(np.float32)
    amax = np.where(all_nan, np.float32(np.nan), amax).astype(np.float32)
    inv6 = np.float32(1.0) / np.float32(6.0)
    with np.errstate(invalid="ignore", over="ignore"):
        sp = (amax * inv6).astype(np.float32)
    sc = np.where(np.isnan(sp), E4M3_MAX, np.minimum(sp, E4M3_MAX)).astype(np.float32)
    s8 = np_e4m3_encode(sc, saturate=True)
    sdec = e4m3_decode_lut()[s8].astype(np.float32)
    with np.errstate(divide="ignore"):
        x_inv = np.where(sdec > 0, np.float32(1.0) / np.where(sdec > 0, sdec, 1), 0).astype(np.float32)
    with np.errstate(invalid="ignore", over="ignore"):
        p = (blk * x_inv[:, :, None]).astype(np.float32)
    c = np.where(np.isnan(p), np.float32(-6.0), np.minimum(np.maximum(p, -6.0), 6.0)).astype(np.float32)
    codes = np_e2m1_encode(c).reshape(M, K)
    xq = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    scales = np.full((nv_sf_bytes(M, K),), 0x38, np.uint8)
    r, g = np.meshgrid(np.arange(M), np.arange(nblk), indexing="ij")
    scales[mx_sf_offset(r, g, ncb)] = s8
    return xq, scales


def np_nv_decode(q: np.ndarray, sc: np.ndarray) -> np.ndarray:
    """float64 values of NVFP4 packed codes [R, K/2] with their tiled scale grid."""
    R, K = q.shape[0], q.shape[1] * 2
    nblk, ncb = K // 16, (K // 16 + 3) // 4
    codes = np.empty((R, K), np.uint8)
    codes[:, 0::2] = q & 15
    codes[:, 1::2] = q >> 4
    dec = np.where(codes & 8, -1.0, 1.0) * E2M1_MAG[codes & 7].astype(np.float64)
    r, g = np.meshgrid(np.arange(R), np.arange(nblk), indexing="ij")
    s = e4m3_decode_lut().astype(np.float64)[sc[mx_sf_offset(r, g, ncb)]]
    return (dec.reshape(R, nblk, 16) * s[:, :, None]).reshape(R, K)


def np_nvfp4_gemm(xq, xs, wq, ws, bias16=None, round_out=False):
    acc = (np_nv_decode(xq, xs) @ np_nv_decode(wq, ws).T).astype(np.float32)
    if bias16 is not None:
        acc = acc + f16_bits_to_f32(np.asarray(bias16, np.uint16))[None, :]
    if round_out:
        acc = acc.astype(np.float16).astype(np.float32)
    return acc
