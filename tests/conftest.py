"""Shared test configuration.

Markers: ``gpu`` -- needs a CUDA device of compute capability 10.x (B200).
The CPU suite (``-m "not gpu"``) covers the oracle, the golden fixtures, the C ABI's
exported symbols and host-side checks, the fake (meta) op implementations and the
multi-rank sharding logic on gloo.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 CUDA device")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O

    O.build()
    return O


@pytest.fixture(scope="session")
def ref_ops():
    """The reference's own compiled CUDA ops (oracle/_ref), or None when not built."""
    from oracle import build_ref

    try:
        return build_ref.load()
    except Exception:  # pragma: no cover - depends on the box
        return None


@pytest.fixture(scope="session")
def capi():
    from fp8linear_b200.capi import CApi

    return CApi()
