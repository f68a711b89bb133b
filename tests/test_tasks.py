"""Synthetic board generators against boards produced by the reference's generators."""

import numpy as np

from ncas_b200 import tasks as T


def test_perfect_mazes_match_reference(golden):
    b = T.maze_boards(4, 19, seed=7)
    assert np.array_equal(b.inputs, golden["maze_inputs"])
    assert np.array_equal(b.targets, golden["maze_targets"])
    assert np.array_equal(b.given, golden["maze_inputs"] != 0)


def test_hard_mazes_match_reference(golden):
    rng = np.random.default_rng(8)
    ins = np.stack([T.hard_maze(30, rng, min_path_len=60, extra_openings=0.10)[0] for _ in range(2)])
    assert np.array_equal(ins, golden["hard_inputs"])


def test_hard_maze_target_is_a_shortest_path():
    rng = np.random.default_rng(0)
    inp, tgt = T.hard_maze(30, rng)
    s = tuple(np.argwhere(inp == T.START)[0])
    g = tuple(np.argwhere(inp == T.GOAL)[0])
    d = T.bfs_dist(inp != T.WALL, s)
    assert int((tgt == T.PATH).sum()) + 2 == d[g] + 1 >= 60


def test_sudoku_symmetry_draws_match_reference(golden):
    rng = np.random.default_rng(21)
    for i in range(3):
        rp, cp, tr, dp = T.sudoku_symmetry(rng)
        assert np.array_equal(rp, golden["sym_rows"][i]) and np.array_equal(cp, golden["sym_cols"][i])
        assert tr == bool(golden["sym_tr"][i]) and np.array_equal(dp, golden["sym_digits"][i])


def test_sudoku_boards_are_valid():
    b = T.sudoku_boards(50, seed=1, clues=(17, 22))
    assert all(T.sudoku_is_solution(t) for t in b.targets)
    n = b.given.sum(axis=(1, 2))
    assert n.min() >= 17 and n.max() <= 22
    assert np.array_equal(b.inputs[b.given], b.targets[b.given]) and (b.inputs[~b.given] == 0).all()
    assert T.sudoku_is_solution(T.canonical_solution())


def test_metrics_exact_and_cell_acc():
    b = T.sudoku_boards(3, seed=2)
    task = T.SudokuTask()
    pred = b.targets.copy()
    pred[1][~b.given[1]] = 0
    m = task.metrics(pred, b)
    assert m["exact"].tolist() == [True, False, True]
    assert m["cell_acc"][1] == 0 and m["valid"][0]


def test_long_rollout_boards_match_reference_generator():
    """The 59x59 boards of the long-rollout fixture (drawn by the reference's
    generate_perfect_maze) come out of our generator for the same seed."""
    from pathlib import Path

    L = np.load(Path(__file__).resolve().parent / "golden" / "long_rollout.npz")
    b = T.maze_boards(len(L["inputs"]), L["inputs"].shape[1], seed=int(L["board_seed"]), goal=False)
    assert np.array_equal(b.inputs, L["inputs"]) and np.array_equal(b.targets, L["targets"])
