"""Op namespace of the native binding (the reference's generated ``_ops.py``).

The reference imports ``ops`` and ``add_op_namespace_prefix`` from a module that its
kernel-builder toolchain generates (torch-ext/fp8linear/layers.py:6). This is the
hand-written equivalent: it loads the in-tree torch binding ``_C.so`` (which links
``libfp8linear_b200.so``) and exposes ``torch.ops.fp8linear_b200``. A missing or
unloadable binding raises ImportError; there is no fallback implementation.
"""
from __future__ import annotations

from pathlib import Path

import torch

NAMESPACE = "fp8linear_b200"
_PKG = Path(__file__).resolve().parent
_BINDING = _PKG / "_C.so"


def _load() -> None:
    if not _BINDING.exists():
        raise ImportError(
            f"fp8linear_b200 native binding not built ({_BINDING} missing); "
            "run `python fp8linear_b200/_build.py`"
        )
    try:
        torch.ops.load_library(str(_BINDING))
    except OSError as e:  # pragma: no cover - depends on the host's CUDA runtime
        raise ImportError(f"cannot load {_BINDING}: {e}") from e


_load()

ops = getattr(torch.ops, NAMESPACE)


def add_op_namespace_prefix(op_name: str) -> str:
    """``"fp8_linear"`` -> ``"fp8linear_b200::fp8_linear"``."""
    return f"{NAMESPACE}::{op_name}"
