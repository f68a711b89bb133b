"""In-tree build of libnca_b200.so for sm_100a (nvcc, no JIT cache).

    python -m ncas_b200.build          # builds ncas_b200/_lib/libnca_b200.so
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent
CSRC = ROOT / "csrc"
OUT = ROOT / "_lib" / "libnca_b200.so"
SOURCES = [CSRC / "api.cu"]
DEPS = SOURCES + [CSRC / "ptx.cuh", CSRC / "step_kernel.cuh", ROOT.parent / "include" / "nca_b200.h"]

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-shared",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    t = OUT.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in DEPS if p.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the CUDA sources into ncas_b200/_lib/libnca_b200.so (skipped when up to date)."""
    if not force and up_to_date():
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, "-o", str(tmp), *map(str, SOURCES)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({' '.join(cmd)}):\n{res.stdout}\n{res.stderr}")
    if verbose:
        print(res.stdout, res.stderr, file=sys.stderr)
    tmp.replace(OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
