"""Generate tests/golden/reference_mx_vectors.npz from the reference's own MXFP8 ops.

Runs on a machine with an sm_100 GPU and the reference ops compiled into oracle/_ref
(``python oracle/build_ref.py`` where the reference tree is present). Writes inputs and
the reference's outputs for:

  * quantize_mxfp8 (csrc/quantize.cu:236-285, kernel :92-131): per-32-element e4m3
    codes and e8m0 block scales in the tiled scale-factor layout (:80-83)
      - ``sweep``: one 32-element block per positive finite bf16 value v, the block's
        largest magnitude being v (scales only: this pins the block-exponent rule for
        every bf16 amax), bf16 rows of K = 1024;
      - ``sweep16``: the same over every positive finite fp16 value;
      - ``edge``: zeros, -0.0, inf, NaN, subnormals, a block whose amax is exactly a
        power of two, values that round past 448 after scaling, K = 96 (three blocks,
        so the fourth scale column of every tile is padding) and M = 14 (padded rows);
      - ``rows``: 24 token rows of the small_cpu workload (K = 1024), codes and scales;
  * mxfp8_gemm (csrc/fp8_gemm.cu:223-345, cuBLASLt VEC32_UE8M0 block-scaled GEMM,
    bias epilogue, fp16 out) on those token rows against 40 MXFP8-quantized weight
    rows of small_cpu with its bias.

Usage: python tests/golden/make_golden_mx.py [out.npz]
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))


def bits16(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def sweep_rows(dtype: torch.dtype, K: int = 1024) -> torch.Tensor:
    """Every positive finite value v of ``dtype`` as the amax of one 32-element block
    (the block also holds -v/2, v/3 and smaller values), packed K/32 blocks per row."""
    if dtype == torch.bfloat16:
        pats = np.arange(0x0001, 0x7F80, dtype=np.uint16)      # positive finite bf16
        vals = torch.from_numpy(pats.view(np.int16)).view(torch.bfloat16).float()
    else:
        pats = np.arange(0x0001, 0x7C00, dtype=np.uint16)      # positive finite fp16
        vals = torch.from_numpy(pats.view(np.int16)).view(torch.float16).float()
    n = vals.numel()
    blocks = torch.zeros(n, 32)
    blocks[:, 0] = vals
    blocks[:, 5] = -vals / 2
    blocks[:, 17] = vals / 3
    blocks[:, 31] = -vals / 7
    per_row = K // 32
    rows = -(-n // per_row)
    pad = rows * per_row - n
    blocks = torch.cat([blocks, torch.zeros(pad, 32)])
    return blocks.reshape(rows, K).to(dtype)


def edge_rows(K: int = 96, M: int = 14) -> torch.Tensor:
    r = np.zeros((M, K), np.float32)
    r[1, :] = -0.0
    r[2, :] = np.resize([np.inf, 1.0, -2.0], K)
    r[3, :] = np.resize([np.nan, 1.0, -3.0, 0.25], K)
    r[4, :] = np.resize([-np.inf, np.nan, 5.0], K)
    r[5, :] = np.resize([1e-40, -3e-39, 2e-41], K)            # bf16 subnormals
    r[6, :] = np.resize([2.0 ** 20, 3.0, -1.0], K)            # amax exactly 2^20
    r[7, :] = np.resize([255.0, 479.0, -511.0, 1.0], K)       # scaled values near 448..512
    r[8, :] = np.resize([3.0e38, -1.0e38, 1.0], K)            # near the bf16 maximum
    r[9, :] = np.resize([1e-30, -1e-31], K)
    r[10, :] = np.linspace(-1000.0, 1000.0, K)
    r[11, :] = np.resize([np.nan], K)                         # all NaN
    r[12, :] = np.resize([0.0, 0.0, 0.0, 7.5], K)
    r[13, :] = np.resize([-448.0, 448.0, 449.0, -464.0], K)
    return torch.from_numpy(r)


def main(out_path: Path) -> None:
    from fp8linear_b200.workloads import WORKLOADS, make_weight, make_x
    from oracle import build_ref

    ref = build_ref.load()
    assert ref is not None, "oracle/_ref/fp8linear_ref.so not built"
    assert torch.cuda.is_available()
    out = {}

    def q(name: str, x: torch.Tensor, keep_codes: bool = True) -> None:
        xq, sc = ref.quantize_mxfp8(x.cuda())
        torch.cuda.synchronize()
        out[f"{name}_x"] = bits16(x)
        out[f"{name}_dtype"] = np.array(0 if x.dtype == torch.bfloat16 else 1)
        out[f"{name}_scales"] = sc.cpu().numpy()
        if keep_codes:
            out[f"{name}_codes"] = xq.cpu().view(torch.uint8).numpy()

    q("sweep", sweep_rows(torch.bfloat16), keep_codes=False)
    q("sweep16", sweep_rows(torch.float16), keep_codes=False)
    q("edge", edge_rows().to(torch.bfloat16))
    q("edge16", edge_rows().clamp(-60000, 60000).to(torch.float16))

    wl = WORKLOADS["small_cpu"]
    x = make_x(wl)[:24]
    w, b = make_weight(wl)
    w = w[:40].contiguous()
    b = b[:40].contiguous()
    q("rows", x)
    xq, xs = ref.quantize_mxfp8(x.cuda())
    wq, ws = ref.quantize_mxfp8(w.cuda())
    y = ref.mxfp8_gemm(xq, xs, wq, ws, b.cuda())
    torch.cuda.synchronize()
    out["gemm_w"] = bits16(w)
    out["gemm_b"] = bits16(b)
    out["gemm_wq"] = wq.cpu().view(torch.uint8).numpy()
    out["gemm_ws"] = ws.cpu().numpy()
    out["gemm_out_f16"] = y.cpu().view(torch.int16).numpy().view(np.uint16)
    np.savez_compressed(out_path, **out)
    print("wrote", out_path, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else Path(__file__).with_name("reference_mx_vectors.npz"))
