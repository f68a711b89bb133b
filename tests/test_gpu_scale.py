"""Parity at the benchmark shapes and at board-shape edges, through the C ABI.

The full benchmark batches (1000 boards x up to 512 trials) are far beyond what the CPU oracle
can step, so these tests use properties that do not depend on size:
  * Philox firing is keyed by (seed, global instance, cell, step), so any single instance of a
    full-size GPU run can be replayed alone by the oracle (inst_offset = its global index);
  * given cells keep their clamp values bit for bit, in every instance, after any number of
    steps (src/nca/model.py:556-566);
  * niche-capped pruning acts per board, so one board of a full-size pruned rollout is replayed
    by the oracle with all its trials.
Board-shape edges: boards wider than a 128-cell tile (the halo window then spans more than three
tiles), single rows and columns, a single cell, all-given and none-given boards."""

import numpy as np
import pytest
import torch

import oracle.nca_oracle as O
from ncas_b200.configs import CONFIGS, boards_for, build, model_config, synthetic_params, task_for
from ncas_b200.rollout import RolloutConfig, rollout
from ncas_b200.tasks import maze_boards

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
TOL = {"bf16": 2e-2, "split": 1e-5}


def oracle_params(task):
    cfg = model_config(task)
    return O.params_from_arrays(synthetic_params(cfg, 0), cfg)


def run_philox(task, precision, inputs, given, K, depth, seed=3, p_fire=0.5, adaptive=False):
    eng = build(task, seed=0, device=DEV, precision=precision).engine()
    N, H, W = inputs.shape
    b = eng.batch_from_boards(inputs, given, K)
    st = eng.new_state(N * K, H * W)
    eng.init_state(st, b)
    x0 = eng.store_nchw(st)
    upd = torch.zeros(N * K, dtype=torch.int32, device=DEV)
    eng.run(st, b, depth, mode="adaptive" if adaptive else "philox", p_fire=p_fire, seed=seed,
            updates=upd)
    x = eng.store_nchw(st)
    eng.check()
    return eng, x0, x, upd


def replay(task, inputs, given, inst, K, depth, channels, seed=3, p_fire=0.5, adaptive=False):
    """The oracle rollout of global instance `inst` (board inst // K) alone."""
    row = inst // K
    fire = "adaptive_philox" if adaptive else "philox"
    return O.rollout(oracle_params(task), inputs[row : row + 1], given[row : row + 1], 1, depth,
                     channels=channels, fire=fire, seed=seed, p_fire=p_fire, inst_offset=inst)


def assert_given_cells_keep_clamp(x0, x, given, K, in_off, c_in):
    """Exact: the input slice of every given cell equals its value after initialisation."""
    g = torch.from_numpy(given.reshape(len(given), -1)).to(DEV).repeat_interleave(K, 0)
    sl0 = x0[:, in_off : in_off + c_in, :]
    sl = x[:, in_off : in_off + c_in, :]
    same = (sl == sl0).all(dim=1)
    assert bool(same[g.bool()].all())


@pytest.mark.parametrize("precision", ["bf16", "split"])
def test_board_wider_than_a_tile_matches_oracle(precision):
    # the 201 x 201 maze of the single-board benchmark config: halo windows span up to 6 tiles
    boards = maze_boards(1, 201, seed=2)
    depth = 3
    _, x0, x, upd = run_philox("maze", precision, boards.inputs, boards.given, 1, depth)
    ref = replay("maze", boards.inputs, boards.given, 0, 1, depth, 32)
    got = x.reshape(1, 32, 201, 201).cpu().numpy()
    assert np.abs(got - ref["x"]).max() <= TOL[precision] * np.abs(ref["x"]).max()
    assert int(upd[0]) == int(ref["updates"][0])
    assert_given_cells_keep_clamp(x0, x, boards.given, 1, 0, 5)


@pytest.mark.parametrize("shape", [(1, 1), (1, 150), (150, 1), (3, 5), (130, 3), (12, 300)])
def test_ragged_board_shapes_match_oracle(shape):
    H, W = shape
    rng = np.random.default_rng(H * 1000 + W)
    inputs = rng.integers(0, 5, size=(3, H, W))
    given = rng.random((3, H, W)) < 0.3
    K, depth = 2, 4
    _, x0, x, upd = run_philox("maze", "split", inputs, given, K, depth)
    p = oracle_params("maze")
    ref = O.rollout(p, inputs, given, K, depth, channels=32, fire="philox", seed=3, p_fire=0.5)
    got = x.reshape(3 * K, 32, H, W).cpu().numpy()
    assert np.abs(got - ref["x"]).max() <= 1e-5 * max(np.abs(ref["x"]).max(), 1e-6)
    assert np.array_equal(upd.cpu().numpy(), ref["updates"])
    assert_given_cells_keep_clamp(x0, x, given, K, 0, 5)


@pytest.mark.parametrize("fraction", [0.0, 1.0])
def test_none_and_all_given(fraction):
    rng = np.random.default_rng(7)
    inputs = rng.integers(0, 10, size=(4, 9, 9))
    given = np.full((4, 9, 9), fraction > 0.5)
    _, x0, x, _ = run_philox("sudoku", "split", inputs, given, 3, 5)
    ref = O.rollout(oracle_params("sudoku"), inputs, given, 3, 5, channels=64, fire="philox",
                    seed=3, p_fire=0.5)
    got = x.reshape(12, 64, 9, 9).cpu().numpy()
    assert np.abs(got - ref["x"]).max() <= 1e-5 * np.abs(ref["x"]).max()
    assert_given_cells_keep_clamp(x0, x, given, 3, 0, 10)


@pytest.mark.parametrize("task,n_small,K,n_big", [("sudoku", 16, 8, 320), ("maze", 8, 4, 240)])
def test_step_ordering_by_tile_counters_equals_grid_barrier(task, n_small, K, n_big):
    """A launch with few tiles per CTA orders its steps by per-tile step counters, a larger one by
    a grid barrier.  The same instances stepped in both (the small batch, then the same boards at
    the front of a batch of more than 8 tiles per SM) give bit-identical states."""
    if task == "sudoku":
        from ncas_b200.tasks import sudoku_boards

        boards = sudoku_boards(n_small, seed=4)
    else:
        boards = maze_boards(n_small, 13, seed=4)
    reps = -(-n_big // n_small)
    big_in = np.concatenate([boards.inputs] * reps)[:n_big]
    big_g = np.concatenate([boards.given] * reps)[:n_big]
    hw = boards.inputs.shape[1] * boards.inputs.shape[2]
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert -(-n_small * K * hw // 128) <= 8 * sms < -(-n_big * K * hw // 128)
    _, _, xa, ua = run_philox(task, "bf16", boards.inputs, boards.given, K, 12, seed=8)
    _, _, xb, ub = run_philox(task, "bf16", big_in, big_g, K, 12, seed=8)
    n = n_small * K
    assert torch.equal(xa, xb[:n]) and torch.equal(ua, ub[:n])


@pytest.mark.parametrize("precision", ["bf16", "split"])
def test_full_cfg2_batch_sampled_instances_match_oracle(precision):
    bc = CONFIGS["cfg2"]  # 1000 sudoku boards x 128 trials
    boards = boards_for(bc, seed=0)
    depth = 6
    _, x0, x, upd = run_philox("sudoku", precision, boards.inputs, boards.given, bc.k, depth)
    n = bc.n_boards * bc.k
    for inst in [0, 1, 127, 128, 64_000, n - 129, n - 1]:
        ref = replay("sudoku", boards.inputs, boards.given, inst, bc.k, depth, 64)
        got = x[inst].reshape(1, 64, 9, 9).cpu().numpy()
        assert np.abs(got - ref["x"]).max() <= TOL[precision] * np.abs(ref["x"]).max(), inst
        assert int(upd[inst]) == int(ref["updates"][0]), inst
    assert_given_cells_keep_clamp(x0, x, boards.given, bc.k, 0, 10)


def test_full_cfg4_batch_adaptive_sampled_instances_match_oracle():
    bc = CONFIGS["cfg4"]  # 1000 sudoku boards x 512 trials, adaptive firing
    boards = boards_for(bc, seed=0)
    depth = 4
    _, x0, x, upd = run_philox("sudoku", "split", boards.inputs, boards.given, bc.k, depth,
                               adaptive=True)
    n = bc.n_boards * bc.k
    for inst in [0, 511, 512, 255_999, n - 1]:
        ref = replay("sudoku", boards.inputs, boards.given, inst, bc.k, depth, 64, adaptive=True)
        got = x[inst].reshape(1, 64, 9, 9).cpu().numpy()
        assert np.abs(got - ref["x"]).max() <= 1e-5 * np.abs(ref["x"]).max(), inst
        assert int(upd[inst]) == int(ref["updates"][0]), inst
    assert_given_cells_keep_clamp(x0, x, boards.given, bc.k, 0, 10)


def test_full_cfg3_pruned_rollout_sampled_boards_match_oracle():
    bc = CONFIGS["cfg3"]  # 1000 hard 30 x 30 mazes x 64 trials, pruning every 20 steps
    boards = boards_for(bc, seed=0)
    depth = 24
    model = build("maze", seed=0, device=DEV, precision="split")
    rc = RolloutConfig(depth=depth, k=bc.k, fire_rate=0.5, max_cells=bc.n_boards * bc.k * bc.hw,
                       pruning={"every": bc.prune_every, "n_cap": bc.n_cap},
                       engine={"precision": "split"})
    res = rollout(model, task_for(bc), boards, rc, seed=5)
    p = oracle_params("maze")
    for r in [0, bc.n_boards - 1]:
        ref = O.rollout(p, boards.inputs[r : r + 1], boards.given[r : r + 1], bc.k, depth,
                        channels=32, fire="philox", seed=5, p_fire=0.5, inst_offset=r * bc.k,
                        prune_every=bc.prune_every, n_cap=bc.n_cap)
        assert np.array_equal(res.pred[r].reshape(bc.k, -1), ref["decoded"].reshape(bc.k, -1)), r
        np.testing.assert_allclose(res.conf[r], ref["conf"], rtol=0, atol=1e-5)
        assert np.array_equal(res.cell_updates[r], ref["updates"].astype(np.float64)), r


def _offset_model(out_offset, precision):
    import dataclasses

    from ncas_b200.model import NCA

    cfg = dataclasses.replace(model_config("sudoku"), out_offset=out_offset)
    params = synthetic_params(cfg, 0)
    m = NCA(cfg, precision=precision)
    with torch.no_grad():
        for name, v in params.items():
            m.get_parameter(name).copy_(torch.from_numpy(v))
    return m.to(DEV).engine(), O.params_from_arrays(params, cfg)


def _adaptive_run(eng, boards, K, depth, chunk):
    b = eng.batch_from_boards(boards.inputs, boards.given, K)
    n = len(boards.inputs) * K
    st = eng.new_state(n, 81)
    eng.init_state(st, b)
    upd = torch.zeros(n, dtype=torch.int32, device=DEV)
    for s0 in range(0, depth, chunk):
        eng.run(st, b, min(chunk, depth - s0), mode="adaptive", seed=3, step0=s0, updates=upd)
    x = eng.store_nchw(st).reshape(n, 64, 9, 9).cpu().numpy()
    eng.check()
    return x, upd.cpu().numpy()


# The confidence warps read the readout slice back from the stored state: a slice across the two
# epilogue channel halves (channels 28..36 of 64) and one ending at the last channel (55..63).
@pytest.mark.parametrize("out_offset", [28, 55])
def test_adaptive_readout_slice_anywhere_in_the_state_matches_oracle(out_offset):
    eng, p = _offset_model(out_offset, "split")
    boards = boards_for(CONFIGS["cfg4"], seed=1, n=3)
    K, depth = 4, 12
    x, upd = _adaptive_run(eng, boards, K, depth, depth)
    ref = O.rollout(p, boards.inputs, boards.given, K, depth, channels=64, fire="adaptive_philox",
                    seed=3, p_fire=0.5)
    assert np.abs(x - ref["x"]).max() <= TOL["split"] * np.abs(ref["x"]).max()
    assert np.array_equal(upd, ref["updates"])


@pytest.mark.parametrize("out_offset", [1, 28, 55])
def test_adaptive_in_kernel_confidence_equals_launch_start_confidence(out_offset):
    # bf16 (hi/lo layout): one launch of 12 steps (the confidence warps give each next step's fire
    # probabilities) against 12 launches of one step (each starts from the probabilities the
    # launch-start kernel computes from the stored state): bit-identical states and counts.
    eng, _ = _offset_model(out_offset, "bf16")
    boards = boards_for(CONFIGS["cfg4"], seed=2, n=3)
    x1, u1 = _adaptive_run(eng, boards, 4, 12, 12)
    x2, u2 = _adaptive_run(eng, boards, 4, 12, 1)
    assert np.array_equal(u1, u2)
    assert np.array_equal(x1, x2)
