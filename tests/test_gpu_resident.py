"""The shared-memory-resident step kernel (bf16 mode below 64 channels): every CTA keeps whole
instances' states in shared memory for all steps of a launch.  It keeps the state as bf16 hi + lo
parts between the steps of a launch (about 16 significant bits, where the streaming kernel keeps
fp32 at 32 channels), so it is checked against the CPU oracle with the bf16 tolerances of the
other tests, against the streaming kernel (the fire decisions, and so the update counts, are
identical; the states agree to the hi + lo rounding), and on the group edges: ragged last groups,
several groups per CTA, boards too large for a group (the streaming kernel then runs)."""

import numpy as np
import pytest
import torch

import oracle.nca_oracle as O
from ncas_b200.configs import build, model_config, synthetic_params
from ncas_b200.tasks import maze_boards

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def run(inputs, given, K, depth, resident, masks=None, seed=5):
    eng = build("maze", seed=0, device=DEV).engine()
    N, H, W = inputs.shape
    b = eng.batch_from_boards(inputs, given, K)
    st = eng.new_state(N * K, H * W)
    eng.init_state(st, b)
    upd = torch.zeros(N * K, dtype=torch.int32, device=DEV)
    if masks is None:
        eng.run(st, b, depth, mode="philox", p_fire=0.5, seed=seed, updates=upd, resident=resident)
    else:
        eng.run(st, b, depth, mode="mask", masks=torch.from_numpy(masks), updates=upd, resident=resident)
    x = eng.store_nchw(st).reshape(N * K, eng.channels, H, W).cpu().numpy()
    r = eng.readout(st, b)
    eng.check()
    return x, upd.cpu().numpy(), r["pred"].reshape(N * K, H, W).cpu().numpy()


def test_resident_matches_oracle_with_external_masks():
    boards = maze_boards(3, 19, seed=31)
    K, D = 2, 24
    B, HW = 3 * K, 19 * 19
    masks = (np.random.default_rng(4).random((D, B, HW)) < 0.5).astype(np.uint8)
    x, upd, dec = run(boards.inputs, boards.given, K, D, True, masks)
    cfg = model_config("maze")
    p = O.params_from_arrays(synthetic_params(cfg, 0), cfg)
    ref = O.rollout(p, boards.inputs, boards.given, K, D, channels=32, masks=masks)
    assert np.abs(x - ref["x"]).max() <= 2e-2 * np.abs(ref["x"]).max()
    assert np.array_equal(upd, masks.reshape(D, B, HW).sum((0, 2)))
    assert (dec != ref["decoded"]).mean() <= 0.01


@pytest.mark.parametrize("n,size,K,depth", [(2, 30, 4, 20),    # cfg3's board shape: one instance per group
                                            (160, 19, 2, 9),   # more groups than SMs: several passes per CTA
                                            (5, 7, 3, 33)])    # small boards, ragged last group
def test_resident_agrees_with_streaming(n, size, K, depth):
    boards = maze_boards(n, size, seed=size + n, hard=size == 30)
    xs, us, ds = run(boards.inputs, boards.given, K, depth, False)
    xr, ur, dr = run(boards.inputs, boards.given, K, depth, True)
    assert np.array_equal(ur, us)  # Philox fire decisions do not depend on the state
    assert np.abs(xr - xs).max() <= 1e-2 * np.abs(xs).max()
    assert (dr != ds).mean() <= 0.01


def test_boards_too_large_for_a_group_run_streaming():
    boards = maze_boards(1, 201, seed=2)
    xs, us, _ = run(boards.inputs, boards.given, 1, 3, False)
    xr, ur, _ = run(boards.inputs, boards.given, 1, 3, True)
    assert np.array_equal(xr, xs) and np.array_equal(ur, us)
