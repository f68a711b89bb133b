"""The reference's trained maze presets (maze_ood: C=16, Hd=128; maze_hard: C=32, Hd=256; learned
perception, wall padding, l2 head) against the reference's own steps of its checkpoints
(tests/golden/presets.npz, made by tests/golden/make_golden.py from the reference): the oracle
here on CPU, the B200 kernels in tests/test_gpu_presets.py."""

import json
from pathlib import Path

import numpy as np
import pytest

import oracle.nca_oracle as O
from ncas_b200.model import NCA, NCAConfig, check_supported

PRESETS = Path(__file__).resolve().parent / "golden" / "presets.npz"
NAMES = ["maze_ood", "maze_hard"]


def load(name):
    g = np.load(PRESETS)
    cfg = NCAConfig.from_dict(json.loads(str(g[f"{name}__config"])))
    w = {k.split("__w__")[1]: g[k] for k in g.files if k.startswith(f"{name}__w__")}
    return g, cfg, w


@pytest.mark.parametrize("name", NAMES)
def test_preset_cell_rule_is_supported_and_loads(name):
    _, cfg, w = load(name)
    check_supported(cfg)
    import torch

    m = NCA(cfg)
    m.load_state_dict({k: torch.from_numpy(v) for k, v in w.items()})
    assert m.cfg.padding == "wall" and m.cfg.head == "l2"


@pytest.mark.parametrize("name", NAMES)
def test_oracle_steps_the_trained_presets_like_the_reference(name):
    g, cfg, w = load(name)
    p = O.params_from_arrays(w, cfg)
    inputs = g[f"{name}__inputs"].astype(np.int64)
    given = g[f"{name}__given"]
    x = g[f"{name}__x0"]
    B, C, H, W = x.shape
    clamp = np.ascontiguousarray(p["embed"][inputs].transpose(0, 3, 1, 2))
    masks = g[f"{name}__masks"]
    for t in range(12):
        x = O.step(x, given[:, None], clamp, masks[t].reshape(B, 1, H, W).astype(np.float32), p)
        if t == 0:
            ref1 = g[f"{name}__x1"]
            assert np.abs(x - ref1).max() <= 1e-5 * np.abs(ref1).max()
    ref = g[f"{name}__x12"]
    assert np.abs(x - ref).max() <= 1e-4 * np.abs(ref).max()
    assert np.array_equal(O.decode_boards(x, given, inputs, p), g[f"{name}__dec12"])
    np.testing.assert_allclose(O.confidence(x, p), g[f"{name}__cconf12"], rtol=0, atol=1e-5)


def test_maze_generators_give_the_presets_boards():
    from ncas_b200.tasks import hard_maze, perfect_maze

    g = np.load(PRESETS)
    r = np.random.default_rng(51)
    for i in range(3):
        inp, tgt = perfect_maze(19, r, goal=False)
        assert np.array_equal(inp, g["maze_ood__inputs"][i]) and np.array_equal(tgt, g["maze_ood__targets"][i])
    r = np.random.default_rng(52)
    for i in range(3):
        inp, tgt = hard_maze(30, r, min_path_len=60, extra_openings=0.10)
        assert np.array_equal(inp, g["maze_hard__inputs"][i]) and np.array_equal(tgt, g["maze_hard__targets"][i])
