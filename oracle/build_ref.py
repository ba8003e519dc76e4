"""Compile the reference's own CUDA ops (drbh/fp8linear) into ``oracle/_ref/``.

Test infrastructure only. The product never imports, links or runs anything
built here; only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
reference leg may load it, and only as the thing compared against.

The reference sources are compiled where they lie (``<ref>/csrc`` and
``<ref>/torch-ext`` of a drbh/fp8linear checkout); nothing is copied into this
repository. ``<ref>`` is ``$FP8LINEAR_REF_ROOT`` when set, else a checkout named
``reference`` next to this repository's root directory. The one
header the reference binding needs and does not ship (``registration.h``, which
its kernel-builder toolchain generates) is replaced by ``oracle/ref_shim``.

Recipe (the reference's nix/kernel-builder build is not used):
  * sources: ``csrc/quantize.cu``, ``csrc/fp8_gemm.cu``, ``torch-ext/torch_binding.cpp``
  * ``TORCH_CUDA_ARCH_LIST=10.0a`` -> ``-gencode arch=compute_100a,code=sm_100a``
  * ``-U__CUDA_NO_HALF_CONVERSIONS__`` and friends, because ``fp8_gemm.cu:77``
    converts ``__half`` to ``float`` implicitly and torch's default flags forbid it
  * link ``-lcublasLt -lcublas``; host compiler /usr/bin/g++ (shared libstdc++)
The result is ``oracle/_ref/fp8linear_ref.so``; loading it with
``torch.ops.load_library`` registers the reference ops under ``torch.ops.fp8linear_ref``.

Usage: ``python oracle/build_ref.py`` (a no-op when the .so is newer than its sources
or when the reference tree is absent, e.g. on a machine that only runs prebuilt files).
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
# a drbh/fp8linear checkout: $FP8LINEAR_REF_ROOT, else <repo>/../reference
REF_ROOT = Path(os.environ.get("FP8LINEAR_REF_ROOT") or HERE.parent.parent / "reference")
OUT_DIR = HERE / "_ref"
NAME = "fp8linear_ref"
SO_PATH = OUT_DIR / f"{NAME}.so"


def sources() -> list[Path]:
    return [
        REF_ROOT / "csrc" / "quantize.cu",
        REF_ROOT / "csrc" / "fp8_gemm.cu",
        REF_ROOT / "torch-ext" / "torch_binding.cpp",
    ]


def up_to_date() -> bool:
    if not SO_PATH.exists():
        return False
    so_m = SO_PATH.stat().st_mtime
    deps = sources() + [HERE / "ref_shim" / "registration.h", Path(__file__)]
    return all((not d.exists()) or d.stat().st_mtime <= so_m for d in deps)


def build(verbose: bool = False) -> Path | None:
    if not all(p.exists() for p in sources()):
        return SO_PATH if SO_PATH.exists() else None
    if up_to_date():
        return SO_PATH
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    # A compiler wrapper that links libstdc++ statically breaks C++ exceptions that
    # torch throws through the extension's frames; use the system g++.
    if Path("/usr/bin/g++").exists():
        os.environ["CXX"] = "/usr/bin/g++"
    os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 4))
    from torch.utils import cpp_extension

    OUT_DIR.mkdir(parents=True, exist_ok=True)
    cpp_extension.load(
        name=NAME,
        sources=[str(p) for p in sources()],
        extra_include_paths=[str(HERE / "ref_shim"), str(REF_ROOT / "torch-ext")],
        extra_cflags=["-O2"],
        extra_cuda_cflags=[
            "-O3",
            "-U__CUDA_NO_HALF_OPERATORS__",
            "-U__CUDA_NO_HALF_CONVERSIONS__",
            "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
            "-U__CUDA_NO_HALF2_OPERATORS__",
        ],
        extra_ldflags=["-L/usr/local/cuda/lib64", "-lcublasLt", "-lcublas"],
        build_directory=str(OUT_DIR),
        is_python_module=False,
        verbose=verbose,
    )
    return SO_PATH


def load():
    """Load the compiled reference ops; returns ``torch.ops.fp8linear_ref`` or None."""
    import torch

    if not SO_PATH.exists():
        return None
    torch.ops.load_library(str(SO_PATH))
    return getattr(torch.ops, NAME)


if __name__ == "__main__":
    p = build(verbose="-v" in sys.argv)
    print(p if p else "reference sources absent; nothing built")
