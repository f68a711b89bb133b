"""ctypes binding of libnca_b200.so (the C ABI declared in include/nca_b200.h).

The shared library is built in-tree by `ncas_b200.build.build()` into `ncas_b200/_lib/`.  There
is no fallback: when the library is missing or does not load, `lib()` raises, and every GPU
entry point of the package fails with that error.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_DIR = Path(__file__).resolve().parent / "_lib"
LIB_PATH = LIB_DIR / "libnca_b200.so"

MAX_OUT = 16
ABI_VERSION = 3  # NCA_B200_ABI_VERSION of include/nca_b200.h

NCA_OK = 0
STATUS_NAMES = {
    0: "NCA_OK",
    1: "NCA_ERR_INVALID",
    2: "NCA_ERR_UNSUPPORTED",
    3: "NCA_ERR_CUDA",
    4: "NCA_ERR_TIMEOUT",
    5: "NCA_ERR_DEVICE",
    6: "NCA_ERR_KERNEL",
    7: "NCA_ERR_SCRATCH",
}
PREC_BF16, PREC_SPLIT = 0, 1
FIRE_MASK, FIRE_PHILOX, FIRE_ADAPTIVE_PHILOX, FIRE_ADAPTIVE_UNIFORM = 0, 1, 2, 3
FIRE_THRESHOLD_PHILOX, FIRE_THRESHOLD_UNIFORM = 4, 5
NOISE_NONE, NOISE_PHILOX, NOISE_EXTERNAL = 0, 1, 2
HEAD_LINEAR, HEAD_L2 = 0, 1


class NcaModelDesc(C.Structure):
    _fields_ = [
        ("channels", C.c_int32),
        ("perception", C.c_int32),
        ("hidden", C.c_int32),
        ("c_in", C.c_int32),
        ("in_offset", C.c_int32),
        ("c_out", C.c_int32),
        ("out_offset", C.c_int32),
        ("n_out", C.c_int32),
        ("fixed_taps", C.c_int32),
        ("taps", (C.c_float * 9) * 4),
        ("head_w", (C.c_float * MAX_OUT) * MAX_OUT),
        ("head_b", C.c_float * MAX_OUT),
        ("out_tokens", C.c_int32 * MAX_OUT),
        ("weights", C.c_void_p),
        ("b1", C.c_void_p),
        ("b2", C.c_void_p),
        ("head_kind", C.c_int32),
        ("pad", C.c_float * 64),
        ("weights_lo", C.c_void_p),
    ]


class NcaBatchDesc(C.Structure):
    _fields_ = [
        ("n_inst", C.c_int32),
        ("height", C.c_int32),
        ("width", C.c_int32),
        ("trials", C.c_int32),
        ("inst_offset", C.c_int64),
        ("given", C.c_void_p),
        ("clamp", C.c_void_p),
        ("inputs", C.c_void_p),
        ("inst_row", C.c_void_p),
        ("inst_id", C.c_void_p),
    ]


class NcaState(C.Structure):
    _fields_ = [
        ("n_inst", C.c_int32),
        ("hw", C.c_int32),
        ("channels", C.c_int32),
        ("precision", C.c_int32),
        ("n_tiles", C.c_int64),
        ("master", C.c_void_p * 2),
        ("mirror", C.c_void_p * 2),
        ("cur", C.c_int32),
        ("clamped", C.c_int32),
        ("tile_steps", C.c_void_p),
        ("fire_p", C.c_void_p),
    ]


class NcaFireDesc(C.Structure):
    _fields_ = [
        ("mode", C.c_int32),
        ("p_fire", C.c_float),
        ("adapt_scale", C.c_float),
        ("adapt_bias", C.c_float),
        ("p_low", C.c_float),
        ("tau", C.c_float),
        ("given_confident", C.c_int32),
        ("seed", C.c_uint64),
        ("step0", C.c_int64),
        ("masks", C.c_void_p),
        ("uniforms", C.c_void_p),
        ("updates", C.c_void_p),
        ("noise_mode", C.c_int32),
        ("noise_p_t", C.c_float),
        ("noise_p_s", C.c_float),
        ("noise_sigma", C.c_float),
        ("noise_until", C.c_int64),
        ("noise", C.c_void_p),
        ("resident", C.c_int32),
    ]


# name -> (restype, argtypes); must match include/nca_b200.h
_P = C.c_void_p
_I = C.c_int32
SIGNATURES = {
    "nca_b200_abi_version": (_I, []),
    "nca_b200_status_string": (C.c_char_p, [_I]),
    "nca_b200_device_info": (_I, [_I, C.POINTER(_I), C.POINTER(_I), C.POINTER(_I)]),
    "nca_b200_weights_bytes": (_I, [_I, _I, _I, C.POINTER(C.c_size_t)]),
    "nca_b200_pack_weights": (_I, [_P, _P, _I, _I, _I, _P]),
    "nca_b200_state_bytes": (_I, [_I, _I, _I, _I, C.POINTER(C.c_size_t)]),
    "nca_b200_state_bind": (_I, [C.POINTER(NcaState), _P, C.c_size_t, _I, _I, _I, _I]),
    "nca_b200_state_init": (
        _I,
        [C.POINTER(NcaState), C.POINTER(NcaModelDesc), C.POINTER(NcaBatchDesc), _P],
    ),
    "nca_b200_state_load_nchw": (_I, [C.POINTER(NcaState), _P, _P]),
    "nca_b200_state_store_nchw": (_I, [C.POINTER(NcaState), _P, _P]),
    "nca_b200_resident_group": (_I, [C.POINTER(NcaModelDesc), _I, _I]),
    "nca_b200_run_steps": (
        _I,
        [
            C.POINTER(NcaModelDesc),
            C.POINTER(NcaBatchDesc),
            C.POINTER(NcaState),
            _I,
            C.POINTER(NcaFireDesc),
            _P,
            _I,
            _P,
        ],
    ),
    "nca_b200_readout": (
        _I,
        [
            C.POINTER(NcaModelDesc),
            C.POINTER(NcaBatchDesc),
            C.POINTER(NcaState),
            _P,
            _P,
            _P,
            _P,
            _P,
            _P,
            _P,
        ],
    ),
    "nca_b200_select": (_I, [_P, _P, _I, _I, _I, _P, _P, _P, _I, _P, _P]),
    "nca_b200_prune_refill": (_I, [_P, _P, _I, _I, _I, _I, _P, _P, _P]),
    "nca_b200_clone": (_I, [C.POINTER(NcaState), _P, _P]),
    "nca_b200_damage": (_I, [C.POINTER(NcaModelDesc), C.POINTER(NcaBatchDesc), C.POINTER(NcaState), _P, _P]),
    "nca_b200_niches": (_I, [_P, _P, _P, _I, _I, _I, _P, _P, _P, _P]),
    "nca_b200_halving": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _P, _P]),
    "nca_b200_gather": (_I, [C.POINTER(NcaState), C.POINTER(NcaState), _P, _P]),
    "nca_b200_ctrl_status": (_I, [_P, C.POINTER(_I), _P]),
    "nca_b200_selftest_timeout": (_I, [_P, _I, _P]),
    "nca_b200_run_steps_static": (
        _I,
        [C.POINTER(NcaModelDesc), C.POINTER(NcaBatchDesc), _I, _P, _P, _I, C.POINTER(NcaFireDesc), _I, _P],
    ),
}

_lib: C.CDLL | None = None


class NcaError(RuntimeError):
    """A non-zero NcaStatus returned by the library."""

    def __init__(self, status: int, where: str, detail: int | None = None):
        self.status = status
        name = STATUS_NAMES.get(status, str(status))
        msg = f"{where}: {name}"
        if _lib is not None:
            msg += f" ({_lib.nca_b200_status_string(status).decode()})"
        if detail:
            msg += f", site {detail}"
        super().__init__(msg)


def lib() -> C.CDLL:
    """Load libnca_b200.so (once) and attach the ctypes signatures."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("NCA_B200_LIB") or LIB_PATH)
    if not path.exists():
        raise RuntimeError(
            f"{path} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'`"
            " (there is no CPU fallback for the B200 rollout)"
        )
    handle = C.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = res
        fn.argtypes = args
    _lib = handle
    return handle


def check(status: int, where: str) -> None:
    if status != NCA_OK:
        raise NcaError(status, where)
