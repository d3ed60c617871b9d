"""Pytest configuration: the ``gpu`` marker and shared helpers for the attention tests."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "attn_golden.npz"
LAYERS_GOLDEN = ROOT / "tests" / "golden" / "layers_golden.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) and the built extension")


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN, allow_pickle=False)


@pytest.fixture(scope="session")
def layers_golden():
    """The reference's RoPE split / merge and energy-network outputs (tests/golden/make_golden.py)."""
    return np.load(LAYERS_GOLDEN, allow_pickle=False)


def golden_case(golden, name: str) -> dict[str, np.ndarray]:
    """The arrays of one whole-stored golden case; bf16 ones are widened to float32 (exact)."""
    meta = golden[f"{name}/meta"]
    dtype = str(meta[0])
    out = {}
    for key in golden.files:
        if not key.startswith(name + "/") or key.endswith("/meta"):
            continue
        arr = golden[key]
        if arr.dtype == np.uint16:
            arr = (arr.astype(np.uint32) << 16).view(np.float32)
        out[key.split("/", 1)[1]] = arr
    out["_dtype"] = dtype
    out["_scale"] = float(meta[1])
    return out


GOLDEN_CASES = ["n1_d64_f32", "n17_d16_f64", "n33_d64_f32", "n81_d64_bf16", "n100_d128_bf16", "n100_d64_bf16"]


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16 (nearest-even) and widen back to float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return (u.astype(np.uint32) << 16).view(np.float32)
