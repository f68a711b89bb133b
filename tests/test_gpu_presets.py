"""The reference's trained maze presets on the B200 kernels (C=16/Hd=128 and C=32/Hd=256
instances, wall padding through the window's padding cell, l2 head in the readout), against the
reference's own steps of its checkpoints (tests/golden/presets.npz).  Split mode carries the
bf16 rounding residual of the fp32 trained weights, so its GEMMs are fp32-accurate."""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from ncas_b200.model import NCA, NCAConfig

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
PRESETS = Path(__file__).resolve().parent / "golden" / "presets.npz"
NAMES = ["maze_ood", "maze_hard"]


def setup(name, precision):
    g = np.load(PRESETS)
    cfg = NCAConfig.from_dict(json.loads(str(g[f"{name}__config"])))
    m = NCA(cfg, precision=precision)
    m.load_state_dict({k.split("__w__")[1]: torch.from_numpy(g[k]) for k in g.files
                       if k.startswith(f"{name}__w__")})
    m = m.to(DEV)
    eng = m.engine()
    inputs, given = g[f"{name}__inputs"].astype(np.int64), g[f"{name}__given"]
    b = eng.batch_from_boards(inputs, given, 1)
    x0 = torch.from_numpy(g[f"{name}__x0"]).to(DEV)
    B, C, H, W = x0.shape
    st = eng.new_state(B, H * W)
    eng.load_nchw(st, x0)
    masks = torch.from_numpy(g[f"{name}__masks"]).to(DEV)
    return g, eng, b, st, masks, (B, C, H, W)


@pytest.mark.parametrize("name", NAMES)
def test_preset_12_steps_split_mode_matches_reference(name):
    g, eng, b, st, masks, shape = setup(name, "split")
    assert eng.wimg_lo is not None  # trained fp32 weights: residual image in use
    eng.run(st, b, 12, mode="mask", masks=masks[:12])
    x = eng.store_nchw(st).reshape(shape).cpu().numpy()
    r = eng.readout(st, b, want_cell_conf=True)
    eng.check()
    ref = g[f"{name}__x12"]
    assert np.abs(x - ref).max() <= 1e-4 * np.abs(ref).max()
    B, C, H, W = shape
    assert np.array_equal(r["pred"].reshape(B, H, W).cpu().numpy(), g[f"{name}__dec12"])
    np.testing.assert_allclose(r["cell_conf"].reshape(B, H, W).cpu().numpy(), g[f"{name}__cconf12"],
                               rtol=0, atol=1e-5)
    np.testing.assert_allclose(r["board_conf"].cpu().numpy(), g[f"{name}__bconf12"], rtol=0, atol=1e-5)


@pytest.mark.parametrize("name", NAMES)
def test_preset_single_step_bf16_mode_within_tolerance(name):
    g, eng, b, st, masks, shape = setup(name, "bf16")
    eng.run(st, b, 1, mode="mask", masks=masks[:1])
    x = eng.store_nchw(st).reshape(shape).cpu().numpy()
    eng.check()
    ref = g[f"{name}__x1"]
    assert np.abs(x - ref).max() <= 2e-2 * np.abs(ref).max()


@pytest.mark.parametrize("name", NAMES)
@pytest.mark.parametrize("precision", ["split", "bf16"])
def test_preset_100_step_rollout_agrees_with_reference(name, precision):
    """Task-level agreement on the trained weights: decoded boards after 100 steps (the maze_ood
    evaluation depth) with the reference's initial states and fire masks."""
    g, eng, b, st, masks, shape = setup(name, precision)
    eng.run(st, b, 100, mode="mask", masks=masks)
    r = eng.readout(st, b)
    eng.check()
    B, C, H, W = shape
    dec = r["pred"].reshape(B, H, W).cpu().numpy()
    ref = g[f"{name}__dec100"]
    if precision == "split":
        assert np.array_equal(dec, ref)
    else:
        assert (dec != ref).mean() <= 0.01  # bf16 GEMMs: cells with near-tied scores may differ
    tg, gv = g[f"{name}__targets"], g[f"{name}__given"]
    solved = [bool((dec[i][~gv[i]] == tg[i][~gv[i]]).all()) for i in range(B)]
    solved_ref = [bool((ref[i][~gv[i]] == tg[i][~gv[i]]).all()) for i in range(B)]
    assert solved == solved_ref


@pytest.mark.parametrize("name", NAMES)
@pytest.mark.parametrize("rule", ["adaptive", "threshold"])
def test_preset_confidence_driven_firing_matches_oracle(name, rule):
    """The confidence-driven fire rules on the trained presets (l2 head): the continuous rule
    p = 0.9 (1 - conf) + 0.1 and the reference's threshold rule (src/nca/model.py:566-593), in
    split mode against the oracle's rollout with the same Philox stream: update counts exact,
    states within the split-mode tolerance."""
    import oracle.nca_oracle as O

    g, eng, _, _, _, _ = setup(name, "split")
    cfg = NCAConfig.from_dict(json.loads(str(g[f"{name}__config"])))
    w = {k.split("__w__")[1]: g[k] for k in g.files if k.startswith(f"{name}__w__")}
    p = O.params_from_arrays(w, cfg)
    inputs, given = g[f"{name}__inputs"].astype(np.int64), g[f"{name}__given"]
    K, D, seed = 2, 10, 5
    n, H, W = inputs.shape
    b = eng.batch_from_boards(inputs, given, K)
    st = eng.new_state(n * K, H * W)
    eng.init_state(st, b)
    upd = torch.zeros(n * K, dtype=torch.int32, device=DEV)
    thr = (0.1, 0.6, True) if rule == "threshold" else None
    eng.run(st, b, D, mode=rule, p_fire=0.5, seed=seed, adaptive=(0.9, 0.1), updates=upd,
            threshold=thr)
    x = eng.store_nchw(st).reshape(n * K, cfg.channels, H, W).cpu().numpy()
    eng.check()
    ref = O.rollout(p, inputs, given, K, D, channels=cfg.channels, fire="adaptive_philox", seed=seed,
                    p_fire=0.5, adaptive=(0.9, 0.1), threshold=thr)
    assert np.array_equal(upd.cpu().numpy(), ref["updates"])
    assert np.abs(x - ref["x"]).max() <= 1e-4 * np.abs(ref["x"]).max()
