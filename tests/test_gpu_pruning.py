"""The reference's Niche-Capped Diversity Pruning (halving at m - 1 checkpoints with batch
compaction, src/nca/pruning.py:22-65, src/nca/rollout.py:154-158, 249-275) through the public
rollout() against the oracle: decoded boards, confidences, update counts and alive flags of every
(board, trial), with pruned trials keeping their values from the checkpoint where they left."""

import numpy as np
import pytest
import torch

import oracle.nca_oracle as O
from ncas_b200.configs import build, model_config, synthetic_params
from ncas_b200.rollout import RolloutConfig, rollout
from ncas_b200.tasks import MazeTask, SudokuTask, maze_boards, sudoku_boards

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def oracle_params(task):
    cfg = model_config(task)
    return O.params_from_arrays(synthetic_params(cfg, 0), cfg)


@pytest.mark.parametrize("task,m,n_cap", [("maze", 4, 2), ("sudoku", 3, 3)])
def test_halving_pruning_with_compaction_matches_oracle(task, m, n_cap):
    if task == "maze":
        boards, K, depth, C, tk = maze_boards(5, 13, seed=6), 16, 24, 32, MazeTask()
    else:
        boards, K, depth, C, tk = sudoku_boards(4, seed=6), 12, 18, 64, SudokuTask()
    model = build(task, seed=0, device=DEV, precision="split")
    rc = RolloutConfig(depth=depth, k=K, fire_rate=0.5, pruning={"m": m, "n_cap": n_cap},
                       record_every=depth // 6, engine={"precision": "split"})
    res = rollout(model, tk, boards, rc, seed=11)
    ref = O.rollout_halving(oracle_params(task), boards.inputs, boards.given, K, depth, channels=C,
                            seed=11, p_fire=0.5, m=m, n_cap=n_cap)
    n = len(boards)
    H, W = boards.shape
    assert np.array_equal(res.alive.reshape(-1), ref["alive"])
    assert np.array_equal(res.pred.reshape(n * K, H, W), ref["decoded"])
    np.testing.assert_allclose(res.conf.reshape(-1), ref["conf"], rtol=0, atol=1e-5)
    assert np.array_equal(res.cell_updates.reshape(-1), ref["updates"].astype(np.float64))
    # every checkpoint halves the alive trials of a board (or keeps what its niches allow)
    assert res.alive.sum(axis=1).max() <= K // 2 ** (m - 1) + 1
    # records: the last record is the final state; a pruned trial's records stop changing
    np.testing.assert_allclose(res.trace_conf[:, :, -1], res.conf, rtol=0, atol=0)
    assert np.array_equal(res.trace_updates[:, :, -1], res.cell_updates)
    dead = ~res.alive
    assert np.all(res.trace_conf[dead][:, -1] == res.trace_conf[dead][:, -2]) or not dead.any()
