"""Generate tests/golden/reference_vectors.npz from the reference's own CUDA ops.

Runs on a machine with an sm_100 GPU and the reference ops compiled into
oracle/_ref (``python oracle/build_ref.py`` where the reference tree is present).
Writes the inputs and the reference's outputs for:

  * quantize_fp8 (csrc/quantize.cu:199-234): 24 token rows of the small_cpu workload
    plus 10 hand-made edge rows (zeros, -0.0, amax exactly 448, e4m3 midpoints,
    subnormal codes, inf, NaN, tiny values), K = 1024, bf16 and fp16;
  * quantize_weight (csrc/quantize.cu:341-366, per-channel branch): 40 weight rows of
    small_cpu plus 4 edge rows, K = 1024;
  * fp8_gemm (csrc/fp8_gemm.cu:139-194, cuBLASLt + dequant kernel, fp16 out) on those
    quantized operands with the small_cpu bias.

Usage: python tests/golden/make_golden.py [out.npz]
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def edge_rows(K: int) -> torch.Tensor:
    from oracle import oracle as O

    lut = O.e4m3_decode_lut()
    fin = np.sort(np.abs(lut[np.isfinite(lut)]))
    mids = ((fin[:-1] + fin[1:]) / 2).astype(np.float32)
    rows = [
        np.zeros(K, np.float32),
        np.full(K, -0.0, np.float32),
        np.concatenate([[448.0], np.linspace(-448, 448, K - 1)]),
        np.resize(mids, K),
        np.resize(np.array([2.0 ** -10, 3 * 2.0 ** -10, 2.0 ** -9, 448.0]), K),
        np.resize(np.array([np.inf, 1.0, -2.0, 0.5]), K),
        np.resize(np.array([np.nan, 1.0, -3.0, 0.25]), K),
        np.resize(np.array([-np.inf, np.nan, 5.0, -5.0]), K),
        np.full(K, 1e-30, np.float32),
        np.resize(np.array([1e4, -3e-3, 7.0, 0.0]), K),
    ]
    return torch.from_numpy(np.stack(rows).astype(np.float32))


def main(out_path: Path) -> None:
    from fp8linear_b200.workloads import WORKLOADS, make_weight, make_x
    from oracle import build_ref

    ref = build_ref.load()
    assert ref is not None, "oracle/_ref/fp8linear_ref.so not built"
    assert torch.cuda.is_available()
    wl = WORKLOADS["small_cpu"]
    K = wl.K
    x = make_x(wl)[:24]
    x_all = torch.cat([x.float(), edge_rows(K)])
    w, b = make_weight(wl)
    w = w[:40]
    b = b[:40]
    w_edge = (torch.randn(4, K, generator=torch.Generator().manual_seed(9)) * 0.02)
    w_edge[0] = 0
    w_edge[1, 5] = 448.0
    w_edge[2] *= 1e-6
    w_edge[3, :8] = torch.tensor([1e-3, -2.5, 0.3, 100.0, -0.0, 7.0, 0.01, -0.01])
    w_all = torch.cat([w, w_edge.bfloat16()])
    b_all = torch.cat([b, torch.zeros(4, dtype=torch.bfloat16)])

    out = {"K": np.int64(K)}
    for name, dt in (("bf16", torch.bfloat16), ("f16", torch.float16)):
        xd = x_all.to(dt).cuda()
        q, s = ref.quantize_fp8(xd)
        out[f"x_{name}"] = bits(xd)
        out[f"xq_{name}"] = q.cpu().view(torch.uint8).numpy()
        out[f"xs_{name}"] = s.cpu().numpy()
    wd = w_all.cuda()
    wq, ws = ref.quantize_weight(wd)
    out["w_bf16"] = bits(wd)
    out["wq"] = wq.cpu().view(torch.uint8).numpy()
    out["ws"] = ws.cpu().numpy()
    out["bias_bf16"] = bits(b_all)
    # GEMM on the finite rows only (the edge rows with inf/NaN make NaN outputs)
    n_fin = 24 + 5
    xq_b = ref.quantize_fp8(x_all[:n_fin].bfloat16().cuda())
    g = ref.fp8_gemm(xq_b[0], xq_b[1], wq, ws, b_all.cuda())
    out["gemm_rows"] = np.int64(n_fin)
    out["gemm_out_f16"] = bits(g)
    np.savez_compressed(out_path, **out)
    print(f"wrote {out_path} ({out_path.stat().st_size} bytes)")


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else Path(__file__).with_name("reference_vectors.npz"))
