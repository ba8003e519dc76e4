"""Generate tests/golden/reference_nv_vectors.npz from the reference's own NVFP4 ops.

Runs on a machine with an sm_100 GPU and the reference ops compiled into oracle/_ref
(``python oracle/build_ref.py`` where the reference tree is present). Writes inputs and
the reference's outputs for:

  * quantize_nvfp4 (csrc/quantize.cu:290-334, kernel :157-194): packed e2m1 codes (two
    per byte) and e4m3 scales per 16 elements in the tiled block-scale layout
      - ``sweep``: one 16-element block per positive finite bf16 value v as the block's
        largest magnitude (with v/2, -v/3, v/5.9, ... beside it), bf16, K = 1024; all
        scales, the codes of every 8th row;
      - ``sweep16``: the same over every positive finite fp16 value;
      - ``edge``: zeros, -0.0, inf, NaN, subnormals, values on the e2m1 rounding
        thresholds, K = 96 (six blocks: the last scale tile is half padding), M = 14;
      - ``rows``: 24 token rows of the small_cpu workload (K = 1024);
  * nvfp4_gemm (csrc/fp8_gemm.cu:347-446, cuBLASLt VEC16_UE4M3 block-scaled e2m1 GEMM,
    bias epilogue, fp16 out) on 128 token rows of small_cpu against 128 NVFP4-quantized
    weight rows with its bias. On B200 with the cuBLASLt of this image the call fails
    (status 15, no algorithm from cublasLtMatmulAlgoGetHeuristic, at every shape tried),
    so the file records the error text under ``gemm_error`` instead of outputs.

Usage: python tests/golden/make_golden_nv.py [out.npz]
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
    if dtype == torch.bfloat16:
        pats = np.arange(0x0001, 0x7F80, dtype=np.uint16)
        vals = torch.from_numpy(pats.view(np.int16)).view(torch.bfloat16).float()
    else:
        pats = np.arange(0x0001, 0x7C00, dtype=np.uint16)
        vals = torch.from_numpy(pats.view(np.int16)).view(torch.float16).float()
    n = vals.numel()
    blocks = torch.zeros(n, 16)
    fr = [1.0, 0.5, -1 / 3, 1 / 5.9, -0.75, 0.25, 1 / 12, -0.125, 0.6, -0.9, 0.375, 0.0,
          -1 / 24, 0.95, -0.51, 0.3]
    for j, c in enumerate(fr):
        blocks[:, j] = vals * c
    per_row = K // 16
    rows = -(-n // per_row)
    blocks = torch.cat([blocks, torch.zeros(rows * per_row - n, 16)])
    return blocks.reshape(rows, K).to(dtype)


def edge_rows(K: int = 96, M: int = 14) -> torch.Tensor:
    r = np.zeros((M, K), np.float32)
    r[1, :] = -0.0
    r[2, :] = np.resize([np.inf, 1.0, -2.0], K)
    r[3, :] = np.resize([np.nan, 1.0, -3.0, 0.25], K)
    r[4, :] = np.resize([-np.inf, np.nan, 5.0], K)
    r[5, :] = np.resize([1e-40, -3e-39, 2e-41], K)
    # e2m1 thresholds with amax 6 (scale 1.0): 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5
    r[6, :] = np.resize([6.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25, -0.75, -1.25,
                         -1.75, -2.5, -3.5, -5.0, 0.2499], K)
    r[7, :] = np.resize([3000.0, 2900.0, -2688.0, 1.0], K)   # amax/6 beyond 448
    r[8, :] = np.resize([3.0e38, -1.0e38, 1.0], K)
    r[9, :] = np.resize([1e-30, -1e-31], K)
    r[10, :] = np.linspace(-1000.0, 1000.0, K)
    r[11, :] = np.resize([np.nan], K)
    r[12, :] = np.resize([0.0, 0.0, 0.0, 7.5, -0.01], K)
    r[13, :] = np.resize([1e-3, 2e-3, -0.0001, 6e-4], K)
    return torch.from_numpy(r)


def main(out_path: Path) -> None:
    from fp8linear_b200.workloads import WORKLOADS, make_weight, make_x
    from oracle import build_ref

    ref = build_ref.load()
    assert ref is not None, "oracle/_ref/fp8linear_ref.so not built"
    assert torch.cuda.is_available()
    out = {}

    def q(name: str, x: torch.Tensor, code_stride: int = 1, keep_x: bool = True) -> None:
        xq, sc = ref.quantize_nvfp4(x.cuda())
        torch.cuda.synchronize()
        if keep_x:  # the sweeps are rebuilt by sweep_rows() instead of stored
            out[f"{name}_x"] = bits16(x)
        out[f"{name}_dtype"] = np.array(0 if x.dtype == torch.bfloat16 else 1)
        out[f"{name}_scales"] = sc.cpu().numpy()
        # codes of every code_stride-th row (keeps the file small; scales are all kept)
        out[f"{name}_codes"] = xq.cpu().numpy()[::code_stride]
        out[f"{name}_code_stride"] = np.array(code_stride)

    q("sweep", sweep_rows(torch.bfloat16), code_stride=8, keep_x=False)
    q("sweep16", sweep_rows(torch.float16), code_stride=8, keep_x=False)
    q("edge", edge_rows().to(torch.bfloat16))
    q("edge16", edge_rows().clamp(-60000, 60000).to(torch.float16))

    wl = WORKLOADS["small_cpu"]
    x = make_x(wl)[:24]
    w, b = make_weight(wl)
    w = w[:128].contiguous()
    b = b[:128].contiguous()
    q("rows", x)
    # the reference's GEMM on 128 x 128 x 1024; only its outcome is kept (on B200 it
    # raises, see the module docstring)
    xg = make_x(wl)[:128].contiguous()
    xq, xs = ref.quantize_nvfp4(xg.cuda())
    wq, ws = ref.quantize_nvfp4(w.cuda())
    try:
        y = ref.nvfp4_gemm(xq, xs, wq, ws, b.cuda())
        torch.cuda.synchronize()
        out["gemm_out_f16"] = y.cpu().view(torch.int16).numpy().view(np.uint16)
    except RuntimeError as e:  # the reference's cuBLASLt call can be unsupported
        out["gemm_error"] = np.array(str(e).splitlines()[0][:200])
    np.savez_compressed(out_path, **out)
    print("wrote", out_path, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else Path(__file__).with_name("reference_nv_vectors.npz"))
