"""The C-ABI library without a GPU: it loads, exports every declared symbol, and its host-side
entry points (weight packing, size queries, argument checks) behave."""

import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

from ncas_b200 import _lib as L
from ncas_b200.build import build
from ncas_b200.configs import bf16_round, model_config
from ncas_b200.model import check_supported

HEADER = Path(__file__).resolve().parents[1] / "include" / "nca_b200.h"


@pytest.fixture(scope="module")
def lib():
    build()
    return L.lib()


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(nca_b200_\w+)\s*\(", text)))


def test_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(L.SIGNATURES), "ctypes signatures and header disagree"


def test_abi_and_status_strings(lib):
    assert lib.nca_b200_abi_version() == L.ABI_VERSION
    assert lib.nca_b200_status_string(4).decode().startswith("a bounded wait")
    assert lib.nca_b200_status_string(0).decode() == "ok"


def unswizzle(img: np.ndarray, rows: int, K: int) -> np.ndarray:
    """Inverse of the 128B-swizzled K-major image, written independently of the C code."""
    out = np.zeros((rows, K), np.uint16)
    for kb in range(K // 64):
        blk = img[kb * rows * 64 : (kb + 1) * rows * 64].reshape(rows, 8, 8)
        for r in range(rows):
            for pos in range(8):
                c = pos ^ (r & 7)
                out[r, kb * 64 + c * 8 : kb * 64 + c * 8 + 8] = blk[r, pos]
    return out


@pytest.mark.parametrize("C_,Hd", [(32, 128), (64, 256)])
def test_pack_weights_layout(lib, C_, Hd):
    P = 4 * C_
    rng = np.random.default_rng(0)
    w1 = rng.standard_normal((Hd, P)).astype(np.float32)
    w2 = rng.standard_normal((C_, Hd)).astype(np.float32)
    n = C.c_size_t(0)
    assert lib.nca_b200_weights_bytes(C_, P, Hd, C.byref(n)) == 0
    assert n.value == 2 * (Hd * P + C_ * Hd)
    img = np.zeros(n.value // 2, np.uint16)
    assert lib.nca_b200_pack_weights(w1.ctypes.data, w2.ctypes.data, C_, P, Hd, img.ctypes.data) == 0
    to16 = lambda a: (bf16_round(a).view(np.uint32) >> 16).astype(np.uint16)  # noqa: E731
    assert np.array_equal(unswizzle(img[: Hd * P], Hd, P), to16(w1))
    assert np.array_equal(unswizzle(img[Hd * P :], C_, Hd), to16(w2))


def test_state_bytes(lib):
    n = C.c_size_t(0)
    assert lib.nca_b200_state_bytes(1000, 81, 64, L.PREC_BF16, C.byref(n)) == 0
    tiles = -(-1000 * 81 // 128)
    lo = tiles * 128 * 64 * 2  # bf16 mode: hi (mirror) and lo bf16 arrays, two buffers each
    hi = tiles * 128 * 64 * 2
    flags = (tiles * 4 + 255) & ~255  # per-tile step counters
    fire_p = tiles * 128 * 4  # per-cell fire probabilities of the confidence rules
    assert n.value == 2 * lo + 2 * hi + flags + fire_p
    assert lib.nca_b200_state_bytes(10, 81, 64, L.PREC_SPLIT, C.byref(n)) == 0
    assert n.value == 2 * (-(-810 // 128) * 128 * 64 * 4 + 255 & ~255) + 256 + 7 * 128 * 4
    assert lib.nca_b200_state_bytes(0, 81, 64, 0, C.byref(n)) == 1


def test_resident_group_sizes(lib):
    def group(C_, Hd, h, w):
        m = L.NcaModelDesc()
        m.channels, m.hidden = C_, Hd
        return lib.nca_b200_resident_group(C.byref(m), h, w)

    # 32 channels: a 30 x 30 maze (900 cells) fits once or more, a 201 x 201 maze does not;
    # 64 channels have no resident kernel
    g30 = group(32, 128, 30, 30)
    assert g30 >= 1
    assert group(32, 128, 201, 201) == 0
    assert group(64, 256, 9, 9) == 0
    # smaller boards pack more instances; 16 channels pack more than 32
    assert group(32, 128, 9, 9) > g30
    assert group(16, 128, 30, 30) >= g30
    assert group(32, 128, 0, 5) == 0


def test_invalid_arguments_are_rejected_without_a_gpu(lib):
    st = L.NcaState()
    assert lib.nca_b200_state_bind(C.byref(st), None, 0, 4, 81, 64, 0) == 1
    assert lib.nca_b200_run_steps(None, None, None, 1, None, None, 0, None) == 1
    assert lib.nca_b200_select(None, None, 0, 1, 1, None, None, None, 0, None, None) == 1
    assert lib.nca_b200_prune_refill(None, None, 1, 8, 4, 2, None, None, None) == 1


def test_unsupported_cell_rules_raise_value_error():
    check_supported(model_config("maze"))
    check_supported(model_config("sudoku"))
    for field, value in [("padding", "wrap"), ("norm_groups", 4), ("head", "cosine"),
                         ("perception", "sobel"), ("embedding", "orthonormal"), ("channels", 128)]:
        cfg = model_config("maze")
        setattr(cfg, field, value)
        with pytest.raises(ValueError):
            check_supported(cfg)


def test_no_cuda_means_a_loud_error():
    import torch

    from ncas_b200.configs import build as build_model

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    m = build_model("maze", device="cpu")
    with pytest.raises(RuntimeError, match="CUDA"):
        m.engine()


def test_torch_operators_are_registered_with_their_schemas(lib):
    """The operator library loads without a GPU and registers every rollout entry point of the C
    ABI as torch.ops.nca_b200.* (the engine calls them)."""
    from ncas_b200._ops import as_bytes, ops

    o = ops()
    want = {
        "state_init": "nca_b200::state_init(Tensor state, Tensor model, Tensor batch) -> ()",
        "run_steps": "nca_b200::run_steps(Tensor model, Tensor batch, Tensor state, int n_steps, "
                     "Tensor fire, Tensor(a!) ctrl, int timeout_ms) -> ()",
        "select": "nca_b200::select(Tensor board_conf, Tensor? alive, int n_boards, int trials, "
                  "int k_limit, Tensor(a!) best_idx, Tensor(b!) best_conf, Tensor? pred, int hw, "
                  "Tensor(c!)? best_pred) -> ()",
        "ctrl_status": "nca_b200::ctrl_status(Tensor(a!) ctrl) -> int[]",
    }
    for name, schema in want.items():
        assert str(getattr(o, name).default._schema) == schema
    for name in ("load_nchw", "store_nchw", "readout", "prune_refill", "clone", "damage", "niches",
                 "halving", "gather"):
        assert hasattr(o, name)
    # a descriptor is a view of the ctypes struct's bytes
    st = L.NcaState()
    v = as_bytes(st)
    assert v.dtype.itemsize == 1 and v.numel() == C.sizeof(L.NcaState)
    v[0] = 7
    assert st.n_inst == 7
