"""Test-time perturbations and the reference's threshold firing rule on the B200 path, against
the oracle: state noise (src/nca/perturb.py:23-40; Philox streams in the kernel, or an external
noise tensor as the reference's torch stream gives it), damage events (src/nca/rollout.py:
206-212) and p_low / tau firing (src/nca/model.py:566-593)."""

import numpy as np
import pytest
import torch

import oracle.nca_oracle as O
from ncas_b200.configs import build, model_config, synthetic_params
from ncas_b200.perturb import circular_masks
from ncas_b200.rollout import RolloutConfig, rollout
from ncas_b200.tasks import MazeTask, SudokuTask, maze_boards, sudoku_boards

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def oracle_params(task):
    cfg = model_config(task)
    return O.params_from_arrays(synthetic_params(cfg, 0), cfg)


def test_philox_noise_matches_oracle():
    boards = sudoku_boards(3, seed=14)
    K, D = 2, 8
    noise = {"p_t": 0.6, "p_s": 0.5, "sigma": 0.05, "until": 6}
    eng = build("sudoku", seed=0, device=DEV, precision="split").engine()
    b = eng.batch_from_boards(boards.inputs, boards.given, K, inst_offset=4)
    st = eng.new_state(3 * K, 81)
    eng.init_state(st, b)
    eng.run(st, b, D, mode="philox", p_fire=0.5, seed=9, noise=noise)
    x = eng.store_nchw(st).reshape(3 * K, 64, 9, 9).cpu().numpy()
    eng.check()
    ref = O.rollout(oracle_params("sudoku"), boards.inputs, boards.given, K, D, channels=64,
                    fire="philox", seed=9, p_fire=0.5, inst_offset=4, noise=noise)
    assert np.abs(x - ref["x"]).max() <= 1e-5 * np.abs(ref["x"]).max()
    # the noise did something: a noise-free run differs
    clean = O.rollout(oracle_params("sudoku"), boards.inputs, boards.given, K, D, channels=64,
                      fire="philox", seed=9, p_fire=0.5, inst_offset=4)
    assert np.abs(clean["x"] - ref["x"]).max() > 1e-3


def test_external_noise_tensor_is_added_before_the_clamp():
    boards = maze_boards(2, 11, seed=3)
    eng = build("maze", seed=0, device=DEV, precision="split").engine()
    b = eng.batch_from_boards(boards.inputs, boards.given, 1)
    st = eng.new_state(2, 121)
    eng.init_state(st, b)
    x0 = eng.store_nchw(st).reshape(2, 32, 11, 11).cpu().numpy()
    g = torch.Generator(device=DEV).manual_seed(2)
    nz = torch.randn((2, 32, 121), generator=g, device=DEV) * 0.1
    masks = (torch.rand((1, 2, 121), generator=g, device=DEV) < 0.5).to(torch.uint8)
    eng.run(st, b, 1, mode="mask", masks=masks, noise={"tensor": nz})
    x = eng.store_nchw(st).reshape(2, 32, 11, 11).cpu().numpy()
    eng.check()
    p = oracle_params("maze")
    _, _, clamp = O.init_state(boards.inputs, boards.given, p, 32)
    xs = np.ascontiguousarray(x0.transpose(0, 2, 3, 1))
    ref = O.step_nhwc(xs, boards.given, np.ascontiguousarray(clamp.transpose(0, 2, 3, 1)),
                      masks.reshape(2, 11, 11).cpu().numpy(), p,
                      nz.reshape(2, 32, 11, 11).permute(0, 2, 3, 1).cpu().numpy())
    ref = ref.transpose(0, 3, 1, 2)
    assert np.abs(x - ref).max() <= 1e-5 * np.abs(ref).max()


def test_damage_event_matches_oracle():
    boards = maze_boards(3, 15, seed=8)
    K, D, t_dmg = 2, 10, 4
    model = build("maze", seed=0, device=DEV, precision="split")
    dmg = {"n": 2, "r_min": 0.1, "r_max": 0.4}
    rc = RolloutConfig(depth=D, k=K, fire_rate=0.5, damage_at=t_dmg, damage=dmg,
                       engine={"precision": "split"})
    res = rollout(model, MazeTask(), boards, rc, seed=21)
    masks = circular_masks(3, 15, 15, 2, 0.1, 0.4, np.random.default_rng(21))
    assert np.array_equal(res.damage_masks, masks) and masks.any()
    ref = O.rollout(oracle_params("maze"), boards.inputs, boards.given, K, D, channels=32,
                    fire="philox", seed=21, p_fire=0.5, damage=(t_dmg, masks))
    assert np.array_equal(res.pred.reshape(3 * K, 15, 15), ref["decoded"])
    np.testing.assert_allclose(res.conf.reshape(-1), ref["conf"], rtol=0, atol=1e-5)


@pytest.mark.parametrize("given_confident", [True, False])
def test_threshold_firing_rule_matches_oracle(given_confident):
    boards = sudoku_boards(3, seed=5)
    K, D = 3, 12
    model = build("sudoku", seed=0, device=DEV, precision="split")
    rc = RolloutConfig(depth=D, k=K, fire_rate=0.5, p_low=0.1, tau=0.12,
                       given_confident=given_confident, engine={"precision": "split"})
    res = rollout(model, SudokuTask(), boards, rc, seed=4)
    ref = O.rollout(oracle_params("sudoku"), boards.inputs, boards.given, K, D, channels=64,
                    fire="adaptive_philox", seed=4, p_fire=0.5,
                    threshold=(0.1, 0.12, given_confident))
    assert np.array_equal(res.cell_updates.reshape(-1), ref["updates"].astype(np.float64))
    assert np.array_equal(res.pred.reshape(3 * K, 9, 9), ref["decoded"])
    np.testing.assert_allclose(res.conf.reshape(-1), ref["conf"], rtol=0, atol=1e-5)


def test_torch_stream_noise_rollout_replays_the_reference_draws():
    """fire='torch': per step the fire draw, then (inside the noise window) the noise draws, on
    one generator in the reference's order (src/nca/rollout.py:213-233); the kernel applies them.
    Replayed here on the same generator and stepped by the oracle."""
    from ncas_b200.perturb import sample_noise

    boards = sudoku_boards(2, seed=9)
    K, D, seed = 2, 6, 13
    noise = {"p_t": 0.7, "p_s": 0.5, "sigma": 0.05, "r": 0.5}
    model = build("sudoku", seed=0, device=DEV, precision="split")
    rc = RolloutConfig(depth=D, k=K, fire_rate=0.5, noise=noise,
                       engine={"precision": "split", "fire": "torch"})
    res = rollout(model, SudokuTask(), boards, rc, seed=seed)

    p = oracle_params("sudoku")
    B = 2 * K
    gen = torch.Generator(device=DEV).manual_seed(seed)
    torch.randn((B, 64, 9, 9), generator=gen, device=DEV)  # the initial-state draw (sigma_init 0)
    x, g4, clamp = O.init_state(np.repeat(boards.inputs, K, 0), np.repeat(boards.given, K, 0), p, 64)
    xs = np.ascontiguousarray(x.transpose(0, 2, 3, 1))
    cl = np.ascontiguousarray(clamp.transpose(0, 2, 3, 1))
    for t in range(D):
        u = torch.rand((B, 1, 9, 9), generator=gen, device=DEV)
        nz = None
        if t < noise["r"] * D:
            n_ = sample_noise(B, 64, 9, 9, noise["p_t"], noise["p_s"], noise["sigma"], gen, DEV)
            nz = None if n_ is None else n_.permute(0, 2, 3, 1).cpu().numpy()
        xs = O.step_nhwc(xs, g4[:, 0], cl, (u < 0.5).reshape(B, 9, 9).cpu().numpy(), p, nz)
    x = np.ascontiguousarray(xs.transpose(0, 3, 1, 2))
    dec = O.decode_boards(x, np.repeat(boards.given, K, 0), np.repeat(boards.inputs, K, 0), p)
    assert np.array_equal(res.pred.reshape(B, 9, 9), dec)
    np.testing.assert_allclose(res.conf.reshape(-1), O.board_confidence(x, p), rtol=0, atol=1e-5)
