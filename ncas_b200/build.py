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
# api.cu holds the entry points and small kernels; each steps_<C>_<HD>.cu the step-kernel
# instances of one model shape (compiled in parallel, then linked into one library)
SOURCES = [CSRC / "api.cu", CSRC / "steps_64_256.cu", CSRC / "steps_32_128.cu",
           CSRC / "steps_16_128.cu", CSRC / "steps_32_256.cu"]
HEADERS = [CSRC / "ptx.cuh", CSRC / "step_kernel.cuh", CSRC / "launch.cuh",
           ROOT.parent / "include" / "nca_b200.h"]
DEPS = SOURCES + HEADERS
# the torch operators over the C ABI (ncas_b200._ops), linked against libnca_b200.so
OPS_SOURCE = CSRC / "torch_ops.cpp"
OPS_OUT = ROOT / "_lib" / "libnca_b200_ops.so"

ARCH_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
]
NVCC_FLAGS = ARCH_FLAGS + ["-shared"]  # the flags of a one-step build (kept for reference)


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def up_to_date() -> bool:
    if not OUT.exists() or not OPS_OUT.exists():
        return False
    t = min(OUT.stat().st_mtime, OPS_OUT.stat().st_mtime)
    return all(p.stat().st_mtime <= t for p in DEPS + [OPS_SOURCE] if p.exists())


def _torch_flags() -> tuple[list[str], list[str]]:
    """Compile and link flags of a C++ file against this interpreter's torch."""
    import torch
    from torch.utils import cpp_extension

    inc = [f"-I{p}" for p in cpp_extension.include_paths()] + ["-I/usr/local/cuda/include"]
    abi = f"-D_GLIBCXX_USE_CXX11_ABI={int(torch.compiled_with_cxx11_abi())}"
    tlib = str(Path(torch.__file__).resolve().parent / "lib")
    libs = [f"-L{tlib}", "-ltorch", "-ltorch_cpu", "-lc10", "-lc10_cuda", "-ltorch_cuda",
            f"-Wl,-rpath,{tlib}"]
    return [abi, *inc], libs


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the CUDA sources into ncas_b200/_lib/libnca_b200.so (skipped when up to date):
    every translation unit to an object in parallel, then one shared-library link."""
    if not force and up_to_date():
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    objdir = ROOT / "_lib" / "obj"
    objdir.mkdir(parents=True, exist_ok=True)
    extra = ["-Xptxas=-v"] if verbose else []
    procs = []
    for src in SOURCES:
        obj = objdir / (src.stem + ".o")
        cmd = [nvcc(), *ARCH_FLAGS, *extra, "-c", "-o", str(obj), str(src)]
        procs.append((cmd, obj, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                                                 text=True)))
    cflags, libs = _torch_flags()
    ops_obj = objdir / "torch_ops.o"
    ops_cmd = ["g++", "-O2", "-std=c++17", "-fPIC", *cflags, "-c", "-o", str(ops_obj), str(OPS_SOURCE)]
    ops_proc = subprocess.Popen(ops_cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
    objs = []
    for cmd, obj, p in procs:
        out, err = p.communicate()
        if p.returncode != 0:
            raise RuntimeError(f"nvcc failed ({' '.join(cmd)}):\n{out}\n{err}")
        if verbose:
            print(out, err, file=sys.stderr)
        objs.append(str(obj))
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(tmp), *objs]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc link failed ({' '.join(cmd)}):\n{res.stdout}\n{res.stderr}")
    tmp.replace(OUT)
    out, err = ops_proc.communicate()
    if ops_proc.returncode != 0:
        raise RuntimeError(f"g++ failed ({' '.join(ops_cmd)}):\n{out}\n{err}")
    tmp = OPS_OUT.with_suffix(".so.tmp")
    cmd = ["g++", "-shared", "-o", str(tmp), str(ops_obj), f"-L{OUT.parent}", "-lnca_b200",
           "-Wl,-rpath,$ORIGIN", *libs]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link of the torch operators failed ({' '.join(cmd)}):\n{res.stdout}\n{res.stderr}")
    tmp.replace(OPS_OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
