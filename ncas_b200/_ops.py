"""The library's entry points as torch operators (torch.ops.nca_b200.*).

`libnca_b200_ops.so` (built in-tree next to libnca_b200.so by `ncas_b200.build.build()`) registers
the C ABI's rollout entry points with torch's dispatcher: they run on torch's current CUDA stream
and raise RuntimeError with the library's status on failure.  The descriptors (NcaModelDesc,
NcaBatchDesc, NcaState, NcaFireDesc) are passed as CPU uint8 views of the ctypes structs
(`as_bytes`), so an operator that advances a state updates the caller's struct.  There is no
fallback: a missing library raises.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import torch

OPS_PATH = Path(__file__).resolve().parent / "_lib" / "libnca_b200_ops.so"
_loaded = False


def ops():
    """torch.ops.nca_b200, with the operator library loaded (once)."""
    global _loaded
    if not _loaded:
        path = Path(os.environ.get("NCA_B200_OPS") or OPS_PATH)
        if not path.exists():
            raise RuntimeError(
                f"{path} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'`"
            )
        from . import _lib

        _lib.lib()  # the C library first (the operator library links against it)
        torch.ops.load_library(str(path))
        _loaded = True
    return torch.ops.nca_b200


def as_bytes(struct: C.Structure) -> torch.Tensor:
    """A CPU uint8 tensor viewing the bytes of a ctypes struct (no copy)."""
    return torch.frombuffer(struct, dtype=torch.uint8)
