"""The CPU oracle against golden vectors recorded from the live reference (no GPU)."""

import numpy as np
import pytest

import oracle.nca_oracle as O
from ncas_b200.configs import bf16_round, model_config, synthetic_params


def params(task):
    cfg = model_config(task)
    return O.params_from_arrays(synthetic_params(cfg, 0), cfg), cfg


def test_synthetic_weights_are_bf16_values():
    cfg = model_config("sudoku")
    d = synthetic_params(cfg, 0)
    w = d["update.fc1.weight"]
    assert np.array_equal(bf16_round(w), w)
    assert 0.015 < float(w.std()) < 0.025


@pytest.mark.parametrize("task", ["maze", "sudoku"])
def test_one_step_matches_reference(golden, task):
    p, cfg = params(task)
    inputs = golden[f"{task}_inputs"].astype(np.int64)
    given = golden["sudoku_given"] if task == "sudoku" else inputs != 0
    K = 2 if task == "sudoku" else 1
    x, g4, clamp = O.init_state(np.repeat(inputs, K, 0), np.repeat(given, K, 0), p, cfg.channels)
    m = golden[f"{task}_masks"][0].reshape(x.shape[0], 1, *x.shape[2:])
    x1 = O.step(x, g4, clamp, m, p)
    np.testing.assert_allclose(x1, golden[f"{task}_x1"], atol=1e-6, rtol=0)


@pytest.mark.parametrize("task", ["maze", "sudoku"])
def test_64_step_rollout_matches_reference(golden, task):
    p, cfg = params(task)
    inputs = golden[f"{task}_inputs"].astype(np.int64)
    given = golden["sudoku_given"] if task == "sudoku" else inputs != 0
    K = 2 if task == "sudoku" else 1
    out = O.rollout(p, inputs, given, K, 64, channels=cfg.channels, masks=golden[f"{task}_masks"])
    np.testing.assert_allclose(out["x"], golden[f"{task}_x64"], atol=2e-5, rtol=0)
    assert np.array_equal(out["decoded"], golden[f"{task}_dec64"])
    np.testing.assert_allclose(O.confidence(out["x"], p), golden[f"{task}_cconf64"], atol=1e-5)
    np.testing.assert_allclose(out["conf"], golden[f"{task}_bconf64"], atol=1e-6)


def test_adaptive_rule_matches_reference(golden):
    p, cfg = params("sudoku")
    u = golden["adapt_u"]
    out = O.rollout(p, golden["sudoku_inputs"].astype(np.int64), golden["sudoku_given"], 2, 16,
                    channels=64, fire="adaptive_uniform", uniforms=u)
    np.testing.assert_allclose(out["x"], golden["adapt_x16"], atol=2e-5, rtol=0)
    assert np.array_equal(out["updates"], golden["adapt_fired"])
    assert np.array_equal(out["decoded"], golden["adapt_dec16"])


def test_zero_fire_mask_is_identity(golden):
    """src/nca/model.py step with an all-zero mask leaves the clamped state unchanged
    (tests/test_model.py:71-79 of the reference)."""
    p, cfg = params("maze")
    inputs = golden["maze_inputs"].astype(np.int64)
    x, g4, clamp = O.init_state(inputs, inputs != 0, p, 32)
    x = x + np.random.default_rng(0).standard_normal(x.shape).astype(np.float32) * 0.1
    x = O.apply_clamp(x, g4, clamp, 0)
    assert np.array_equal(O.step(x, g4, clamp, np.zeros((4, 1, 19, 19)), p), x)


def test_given_cells_stay_clamped(golden):
    p, cfg = params("sudoku")
    out = O.rollout(p, golden["sudoku_inputs"].astype(np.int64), golden["sudoku_given"], 2, 8,
                    channels=64, masks=np.ones((8, 8, 81), np.uint8))
    x = out["x"]
    g = np.repeat(golden["sudoku_given"], 2, 0)
    toks = np.repeat(golden["sudoku_inputs"], 2, 0).astype(np.int64)
    emb = p["embed"][toks]  # (B, 9, 9, 10)
    assert np.array_equal(x[:, :10].transpose(0, 2, 3, 1)[g], emb[g])


def test_fixed_perception_equals_block_diagonal_conv():
    """KernelPerception = dense conv with block-diagonal weights (tests/test_model.py:34-49)."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((2, 5, 7, 7)).astype(np.float32)
    taps = rng.standard_normal((3, 9)).astype(np.float32)
    z = O.perceive(x, taps)
    xp = np.pad(x, ((0, 0), (0, 0), (1, 1), (1, 1)))
    for k in range(3):
        for c in range(5):
            ref = sum(taps[k, n] * xp[:, c, n // 3 : n // 3 + 7, n % 3 : n % 3 + 7] for n in range(9))
            np.testing.assert_allclose(z[:, k * 5 + c], ref, atol=1e-5)


# Known-answer vectors of Philox4x32-10 (Salmon et al., SC'11; the Random123 distribution's
# kat_vectors file): counter, key -> output.
PHILOX_KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


@pytest.mark.parametrize("ctr,key,want", PHILOX_KAT)
def test_philox_known_answers(ctr, key, want):
    out = O.philox4x32_10([np.array([c], np.uint64) for c in ctr], key)
    assert tuple(int(o[0]) for o in out) == want


def test_philox_uniform_range_and_rate():
    u = O.philox_uniform(123, np.arange(64)[:, None], np.arange(900)[None, :], 7)
    assert u.dtype == np.float32 and u.min() >= 0 and u.max() < 1
    assert abs(float((u < 0.5).mean()) - 0.5) < 0.01


def test_rollout_halving_halves_alive_trials_per_checkpoint():
    from ncas_b200.tasks import maze_boards

    cfg = model_config("maze")
    p = O.params_from_arrays(synthetic_params(cfg, 0), cfg)
    boards = maze_boards(3, 9, seed=2)
    out = O.rollout_halving(p, boards.inputs, boards.given, 8, 8, channels=32, seed=1, m=2, n_cap=8)
    alive = out["alive"].reshape(3, 8)
    # one checkpoint: floor(8 / 2) survivors per board (n_cap large enough to never bind)
    assert np.array_equal(alive.sum(axis=1), [4, 4, 4])
    assert out["decoded"].shape == (24, 9, 9) and np.all(out["updates"] > 0)


def test_torch_cpu_port_matches_numpy_oracle():
    """oracle/torch_cpu.py (the CPU baseline, computed with the reference's torch operators)
    steps exactly like the numpy oracle on the same masks, maze and sudoku."""
    import torch

    import oracle.torch_cpu as TC
    from ncas_b200.configs import model_config, synthetic_params
    from ncas_b200.tasks import maze_boards, sudoku_boards

    for task, boards in (("maze", maze_boards(2, 19, seed=4)), ("sudoku", sudoku_boards(3, seed=4))):
        cfg = model_config(task)
        p = O.params_from_arrays(synthetic_params(cfg, 0), cfg)
        m = TC.TorchCpuNca(p, cfg.channels)
        x, g4, cl = TC.init_state(boards.inputs, boards.given, 2, cfg.channels, m.c_in, m.in_off)
        for t in range(3):
            fire = (torch.rand((x.shape[0], 1, *x.shape[2:]), generator=torch.Generator().manual_seed(t)) < 0.5).float()
            want = O.step(x.numpy(), g4.numpy(), cl.numpy(), fire.numpy(), p)
            with torch.no_grad():
                x = m.step(x, g4, cl, fire)
            np.testing.assert_allclose(x.numpy(), want, rtol=1e-5, atol=1e-6)
