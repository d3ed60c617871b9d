"""Build ``libebr_attn.so`` in-tree with nvcc for sm_100a (``python -m ebr_b200.build``).

The library is one translation unit (``csrc/capi.cu`` includes the kernel headers), linked against the static CUDA
runtime so it carries no dependency on a particular ``libcudart`` on the GPU box.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT = PKG / "libebr_attn.so"
ROOT = PKG.parent

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-shared",
    "-Xcompiler",
    "-fPIC",
    "-cudart",
    "static",
    "-diag-suppress",
    "1886",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "ebr_attn.h", ROOT / "include" / "ebr_layers.h"]


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    mtime = OUT.stat().st_mtime
    return all(p.stat().st_mtime <= mtime for p in sources())


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    if not force and up_to_date():
        return OUT
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, *(extra or []), "-o", str(tmp), str(CSRC / "capi.cu")]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    tmp.replace(OUT)
    return OUT


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose=True, extra=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None)
    print(p)
