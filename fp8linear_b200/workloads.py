"""Synthetic FLUX-shaped workloads (seeded) for tests and benchmarks.

FLUX.1-dev weights and activations are not available offline, so seeded synthetic
tensors with the same shapes and value distributions stand in for them. The shapes
are the FLUX linears the reference's own hardware scripts time
(scripts/mxfp8_check.py:19-25 of the reference):

  small_cpu      M=256,   K=1024  -> N=1024    x ~ N(0,1), 1% channels x20
  flux_qkv       M=4608,  K=3072  -> N=9216    x ~ N(0,1), 0.5% channels x50
  flux_fc1       M=4608,  K=3072  -> N=12288   x ~ N(0,1), 0.5% channels x50
  flux_fc2       M=4608,  K=12288 -> N=3072    x ~ GELU(N(0,1))
  flux_linear1   M=18432, K=3072  -> N=21504   x ~ N(0,1), 0.5% channels x50
  flux_linear2   M=18432, K=15360 -> N=3072    x ~ N(0,1), 0.5% channels x50
  sweep_M<m>     M=m,     K=3072  -> N=3072    x ~ N(0,1), m in SWEEP_M
  flux_linear2_rank8  M=2304, K=15360 -> N=3072  linear2 rows of one of 8 GPUs splitting
                 the 18432 (batch-4 single-stream block) rows, as flux_linear2

Weights are N(0, 0.02) in bf16, bias N(0, 0.02) in bf16. Each workload uses its own
generator seeded with ``seed``; values are drawn on ``gen_device`` so the same
(workload, seed, gen_device) always yields the same bytes.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

SWEEP_M = (1, 16, 128, 1024, 4096, 16384, 65536)


@dataclass(frozen=True)
class Workload:
    name: str
    M: int
    K: int
    N: int
    dist: str = "normal"  # "normal" | "gelu"
    outlier_frac: float = 0.0
    outlier_scale: float = 1.0

    @property
    def flops(self) -> int:
        return 2 * self.M * self.N * self.K

    @property
    def quant_bytes(self) -> int:
        """Algorithmic bytes of the per-token quantizer: read 2MK, write MK + 4M."""
        return self.M * (3 * self.K + 4)

    @property
    def gemm_bytes(self) -> int:
        """Compulsory bytes of the fused GEMM: codes in, scales, bias, bf16 out."""
        return self.M * self.K + self.N * self.K + 4 * self.M + 4 * self.N + 2 * self.N \
            + 2 * self.M * self.N


def _build() -> dict[str, Workload]:
    w = [
        Workload("small_cpu", 256, 1024, 1024, "normal", 0.01, 20.0),
        Workload("flux_qkv", 4608, 3072, 9216, "normal", 0.005, 50.0),
        Workload("flux_fc1", 4608, 3072, 12288, "normal", 0.005, 50.0),
        Workload("flux_fc2", 4608, 12288, 3072, "gelu"),
        Workload("flux_linear1", 18432, 3072, 21504, "normal", 0.005, 50.0),
        Workload("flux_linear2", 18432, 15360, 3072, "normal", 0.005, 50.0),
    ]
    w += [Workload(f"sweep_M{m}", m, 3072, 3072) for m in SWEEP_M]
    w.append(Workload("flux_linear2_rank8", 18432 // 8, 15360, 3072, "normal", 0.005, 50.0))
    return {x.name: x for x in w}


WORKLOADS = _build()


def make_x(wl: Workload, M: int | None = None, seed: int = 0, gen_device: str = "cpu",
           dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """Activations [M, K] for ``wl`` (M defaults to wl.M), on ``gen_device``."""
    M = wl.M if M is None else M
    g = torch.Generator(device=gen_device)
    g.manual_seed(seed)
    x = torch.randn(M, wl.K, generator=g, device=gen_device, dtype=torch.float32)
    if wl.dist == "gelu":
        x = torch.nn.functional.gelu(x)
    if wl.outlier_frac > 0:
        n_out = int(round(wl.outlier_frac * wl.K))
        idx = torch.randperm(wl.K, generator=g, device=gen_device)[:n_out]
        x[:, idx] *= wl.outlier_scale
    return x.to(dtype)


def make_weight(wl: Workload, seed: int = 0, gen_device: str = "cpu",
                dtype: torch.dtype = torch.bfloat16):
    """(w [N, K], bias [N]) for ``wl``: N(0, 0.02) each, in ``dtype``."""
    g = torch.Generator(device=gen_device)
    g.manual_seed(seed + 1)
    w = (torch.randn(wl.N, wl.K, generator=g, device=gen_device) * 0.02).to(dtype)
    b = (torch.randn(wl.N, generator=g, device=gen_device) * 0.02).to(dtype)
    return w, b
