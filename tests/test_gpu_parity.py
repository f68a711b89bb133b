"""Parity of the CUDA path (through the C ABI) with the reference's golden vectors and the CPU
oracle.  Tolerances (north star): single step within 2e-2 max relative error in bf16 mode;
decoded argmax after 64 steps bit-exact in split mode (bf16 hi+lo GEMM operands); selection and
pruning bit-exact given identical confidences."""

import ctypes as C

import numpy as np
import pytest
import torch

import oracle.nca_oracle as O
from ncas_b200 import _lib as L
from ncas_b200.configs import build, model_config, synthetic_params
from ncas_b200.tasks import maze_boards, sudoku_boards

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def oracle_params(task):
    cfg = model_config(task)
    return O.params_from_arrays(synthetic_params(cfg, 0), cfg), cfg


def golden_case(golden, task):
    inputs = golden[f"{task}_inputs"].astype(np.int64)
    given = golden["sudoku_given"] if task == "sudoku" else inputs != 0
    K = 2 if task == "sudoku" else 1
    return inputs, given, K


def run_kernel(task, precision, inputs, given, K, masks, steps=None, per_launch=None):
    """Kernel rollout with external masks; returns (engine, state, batch, x (B,C,H,W))."""
    m = build(task, seed=0, device=DEV, precision=precision)
    eng = m.engine()
    B = len(inputs) * K
    H, W = inputs.shape[1:]
    b = eng.batch_from_boards(inputs, given, K)
    st = eng.new_state(B, H * W)
    eng.init_state(st, b)
    steps = masks.shape[0] if steps is None else steps
    per = steps if per_launch is None else per_launch
    mk = torch.from_numpy(masks.reshape(masks.shape[0], B, H * W).astype(np.uint8))
    for t0 in range(0, steps, per):
        eng.run(st, b, min(per, steps - t0), mode="mask", masks=mk[t0 : t0 + per], step0=t0)
    x = eng.store_nchw(st).reshape(B, eng.channels, H, W).cpu().numpy()
    eng.check()
    return eng, st, b, x


@pytest.mark.parametrize("task", ["maze", "sudoku"])
@pytest.mark.parametrize("precision,tol", [("bf16", 2e-2), ("split", 1e-5)])
def test_single_step_against_reference(golden, task, precision, tol):
    inputs, given, K = golden_case(golden, task)
    _, _, _, x1 = run_kernel(task, precision, inputs, given, K, golden[f"{task}_masks"][:1])
    ref = golden[f"{task}_x1"]
    rel = np.abs(x1 - ref).max() / np.abs(ref).max()
    assert rel <= tol, f"max relative error {rel:.3e}"
    # the update itself (x1 - x0) is also close in relative terms
    x0 = O.init_state(np.repeat(inputs, K, 0), np.repeat(given, K, 0), oracle_params(task)[0],
                      32 if task == "maze" else 64)[0]
    d_ref, d = ref - x0, x1 - x0
    assert np.abs(d - d_ref).max() <= (5e-2 if precision == "bf16" else 1e-4) * np.abs(d_ref).max()


@pytest.mark.parametrize("task", ["maze", "sudoku"])
def test_64_step_argmax_bit_exact_split(golden, task):
    inputs, given, K = golden_case(golden, task)
    eng, st, b, x = run_kernel(task, "split", inputs, given, K, golden[f"{task}_masks"])
    r = eng.readout(st, b, want_cell_conf=True)
    H, W = inputs.shape[1:]
    dec = r["pred"].reshape(-1, H, W).cpu().numpy()
    assert np.array_equal(dec, golden[f"{task}_dec64"])
    np.testing.assert_allclose(x, golden[f"{task}_x64"], atol=2e-5, rtol=0)
    np.testing.assert_allclose(r["board_conf"].cpu().numpy(), golden[f"{task}_bconf64"], atol=1e-5)


@pytest.mark.parametrize("task", ["maze", "sudoku"])
def test_64_step_argmax_bf16_flips_only_at_near_ties(golden, task):
    inputs, given, K = golden_case(golden, task)
    eng, st, b, x = run_kernel(task, "bf16", inputs, given, K, golden[f"{task}_masks"])
    H, W = inputs.shape[1:]
    dec = eng.readout(st, b)["pred"].reshape(-1, H, W).cpu().numpy()
    p, _ = oracle_params(task)
    s = O.scores(golden[f"{task}_x64"], p)
    top2 = np.sort(s, axis=1)[:, -2:]
    margin = top2[:, 1] - top2[:, 0]
    flips = dec != golden[f"{task}_dec64"]
    mutable = ~np.repeat(given, K, 0)
    print(f"{task} bf16: {int(flips.sum())} flips of {int(mutable.sum())} mutable cells")
    assert flips.sum() <= 0.01 * mutable.sum()
    if flips.any():
        assert margin[flips].max() < 2e-3 * np.abs(s).max()


@pytest.mark.parametrize("precision", ["bf16", "split"])
def test_readout_matches_reference(golden, precision):
    task = "sudoku"
    inputs, given, K = golden_case(golden, task)
    m = build(task, seed=0, device=DEV, precision=precision)
    eng = m.engine()
    b = eng.batch_from_boards(inputs, given, K)
    st = eng.new_state(8, 81)
    eng.load_nchw(st, torch.from_numpy(golden["sudoku_x64"]))
    tg = torch.from_numpy(golden["sudoku_targets"])  # per board row, shared by its K trials
    r = eng.readout(st, b, targets=tg, want_cell_conf=True)
    eng.check()
    assert np.array_equal(r["pred"].reshape(8, 9, 9).cpu().numpy(), golden["sudoku_dec64"])
    np.testing.assert_allclose(r["cell_conf"].reshape(8, 9, 9).cpu().numpy(), golden["sudoku_cconf64"], atol=1e-6)
    np.testing.assert_allclose(r["board_conf"].cpu().numpy(), golden["sudoku_bconf64"], atol=1e-6)
    dec = golden["sudoku_dec64"].astype(np.int64)
    mut = ~np.repeat(given, K, 0)
    tgt = np.repeat(golden["sudoku_targets"], K, 0)
    acc = ((dec == tgt) & mut).sum((1, 2)) / np.maximum(mut.sum((1, 2)), 1)
    np.testing.assert_allclose(r["cell_acc"].cpu().numpy(), acc, atol=1e-6)


def test_adaptive_firing_matches_reference(golden):
    inputs, given, K = golden_case(golden, "sudoku")
    m = build("sudoku", seed=0, device=DEV, precision="split")
    eng = m.engine()
    b = eng.batch_from_boards(inputs, given, K)
    st = eng.new_state(8, 81)
    eng.init_state(st, b)
    upd = torch.zeros(8, dtype=torch.int32, device=DEV)
    eng.run(st, b, 16, mode="adaptive_uniform", uniforms=torch.from_numpy(golden["adapt_u"]).reshape(16, 8, 81),
            adaptive=(0.9, 0.1), updates=upd)
    x = eng.store_nchw(st).reshape(8, 64, 9, 9).cpu().numpy()
    eng.check()
    assert np.array_equal(upd.cpu().numpy(), golden["adapt_fired"])
    np.testing.assert_allclose(x, golden["adapt_x16"], atol=2e-5, rtol=0)


@pytest.mark.parametrize("precision", ["bf16", "split"])
def test_philox_stream_matches_oracle(precision):
    boards = maze_boards(3, 19, seed=4)
    K, D = 2, 6
    m = build("maze", seed=0, device=DEV, precision=precision)
    eng = m.engine()
    b = eng.batch_from_boards(boards.inputs, boards.given, K, inst_offset=10)
    st = eng.new_state(6, 361)
    eng.init_state(st, b)
    upd = torch.zeros(6, dtype=torch.int32, device=DEV)
    eng.run(st, b, D, mode="philox", p_fire=0.5, seed=77, updates=upd)
    x = eng.store_nchw(st).reshape(6, 32, 19, 19).cpu().numpy()
    eng.check()
    p, _ = oracle_params("maze")
    ref = O.rollout(p, boards.inputs, boards.given, K, D, channels=32, fire="philox", seed=77,
                    p_fire=0.5, inst_offset=10)
    assert np.array_equal(upd.cpu().numpy(), ref["updates"])
    tol = 1e-5 if precision == "split" else 2e-2
    assert np.abs(x - ref["x"]).max() <= tol * np.abs(ref["x"]).max()


def test_multi_step_launch_equals_single_steps():
    boards = sudoku_boards(5, seed=9)
    masks = (np.random.default_rng(3).random((12, 15, 81)) < 0.5).astype(np.uint8)
    _, _, _, xa = run_kernel("sudoku", "bf16", boards.inputs, boards.given, 3, masks)
    _, _, _, xb = run_kernel("sudoku", "bf16", boards.inputs, boards.given, 3, masks, per_launch=1)
    _, _, _, xc = run_kernel("sudoku", "bf16", boards.inputs, boards.given, 3, masks, per_launch=5)
    assert np.array_equal(xa, xb) and np.array_equal(xa, xc)


def test_deterministic():
    boards = maze_boards(2, 19, seed=1)
    masks = (np.random.default_rng(5).random((10, 2, 361)) < 0.5).astype(np.uint8)
    xa = run_kernel("maze", "bf16", boards.inputs, boards.given, 1, masks)[3]
    xb = run_kernel("maze", "bf16", boards.inputs, boards.given, 1, masks)[3]
    assert np.array_equal(xa, xb)


def test_select_matches_oracle():
    rng = np.random.default_rng(0)
    N, K = 300, 64
    conf = rng.random((N, K)).astype(np.float32)
    conf[:, 5] = conf[:, 9]  # ties: first index wins
    alive = rng.random((N, K)) < 0.7
    alive[7] = False  # no alive trial: index 0, like np.argmax over -inf
    # diverged trials: np.argmax returns the first alive NaN; a dead NaN is ignored
    conf[11, [3, 40]] = np.nan
    alive[11, [3, 40]] = True
    conf[12, 2] = np.nan
    alive[12, 2] = False
    pred = rng.integers(0, 10, (N * K, 81), dtype=np.uint8)
    m = build("sudoku", seed=0, device=DEV)
    eng = m.engine()
    for k in (1, 7, 64):
        idx, best, bp = eng.select(torch.from_numpy(conf).to(DEV).reshape(-1), N, K, k_limit=k,
                                   alive=torch.from_numpy(alive).reshape(-1), pred=torch.from_numpy(pred).to(DEV), hw=81)
        want = O.best_trial(conf, alive, k)
        assert np.array_equal(idx.cpu().numpy(), want)
        assert np.array_equal(bp.cpu().numpy(), pred.reshape(N, K, 81)[np.arange(N), want])
        got = best.cpu().numpy()
        ref = np.where(alive[:, :k], conf[:, :k], -np.inf)[np.arange(N), want]
        assert np.array_equal(got, ref.astype(np.float32), equal_nan=True)


def test_prune_refill_matches_oracle():
    rng = np.random.default_rng(1)
    N, K, HW = 40, 64, 900
    base = rng.integers(0, 2, (N, 6, HW), dtype=np.uint8)
    dec = base[np.arange(N)[:, None], rng.integers(0, 6, (N, K))]  # 6 candidate grids per board
    conf = rng.random((N, K)).astype(np.float32)
    conf[:, 3] = conf[:, 4]
    m = build("maze", seed=0, device=DEV)
    eng = m.engine()
    st = eng.new_state(N * K, HW)
    src, kept = eng.prune_refill(st, torch.from_numpy(dec.reshape(N * K, HW)).to(DEV),
                                 torch.from_numpy(conf.reshape(-1)).to(DEV), N, K, 2)
    want_src, want_kept = O.niche_cap_refill(dec, conf, 2)
    assert np.array_equal(kept.cpu().numpy().reshape(N, K).astype(bool), want_kept)
    assert np.array_equal(src.cpu().numpy().reshape(N, K), want_src + np.arange(N)[:, None] * K)


def test_clone_copies_states():
    boards = maze_boards(2, 19, seed=2)
    masks = (np.random.default_rng(6).random((3, 8, 361)) < 0.5).astype(np.uint8)
    eng, st, b, x = run_kernel("maze", "bf16", boards.inputs, boards.given, 4, masks)
    src = torch.tensor([0, 0, 2, 2, 4, 7, 6, 7], dtype=torch.int32, device=DEV)  # sources map to themselves
    L.check(L.lib().nca_b200_clone(C.byref(st.st), src.data_ptr(), eng._s()), "clone")
    y = eng.store_nchw(st).reshape(8, 32, 19, 19).cpu().numpy()
    assert np.array_equal(y, x[src.cpu().numpy()])


@pytest.mark.parametrize("precision", ["bf16", "split"])
def test_nchw_roundtrip_and_ragged_batch(precision):
    m = build("sudoku", seed=0, device=DEV, precision=precision)
    eng = m.engine()
    x = torch.randn(7, 64, 9, 9, device=DEV)  # 567 cells: a partial last tile
    st = eng.new_state(7, 81)
    eng.load_nchw(st, x)
    y = eng.store_nchw(st).reshape(7, 64, 9, 9)
    if precision == "split":
        assert torch.equal(y, x)  # fp32 state
    else:
        # bf16 mode keeps x as hi = bf16(x) plus lo = bf16(x - hi): about 16 significant bits
        assert bool(((y - x).abs() <= x.abs() * 2.0 ** -15).all())


def test_drop_in_step_and_blocks_match_oracle():
    from ncas_b200.engine import B200RolloutBlocks

    boards = maze_boards(3, 19, seed=5)
    m = build("maze", seed=0, device=DEV, precision="split")
    inputs = torch.from_numpy(boards.inputs).to(DEV)
    given = torch.from_numpy(boards.given).to(DEV)
    x, g4, clamp = m.init_state(inputs, given)
    fm = (torch.rand((3, 1, 19, 19), device=DEV) < 0.5).float()
    y = m.step(x, g4, clamp, fm)
    p, _ = oracle_params("maze")
    ref = O.step(x.cpu().numpy(), g4.cpu().numpy(), clamp.cpu().numpy(), fm.cpu().numpy(), p)
    np.testing.assert_allclose(y.cpu().numpy(), ref, atol=1e-6, rtol=0)
    blocks = B200RolloutBlocks(m, {"precision": "split"})
    fires = [(torch.rand((3, 1, 19, 19), device=DEV) < 0.5).float() for _ in range(4)]
    z = blocks(x, g4, clamp, fires, [None] * 4)
    ref = x.cpu().numpy()
    for f in fires:
        ref = O.step(ref, g4.cpu().numpy(), clamp.cpu().numpy(), f.cpu().numpy(), p)
    np.testing.assert_allclose(z.cpu().numpy(), ref, atol=1e-5, rtol=0)
    dec = m.decode(z)
    assert torch.equal(dec.cpu(), torch.from_numpy(O.decode(z.cpu().numpy(), p)))


def test_bounded_wait_reports_timeout_and_context_survives():
    ctrl = torch.zeros(4, dtype=torch.int32, device=DEV)
    s = L.lib().nca_b200_selftest_timeout(ctrl.data_ptr(), 50, torch.cuda.current_stream().cuda_stream)
    assert s == 4  # NCA_ERR_TIMEOUT
    boards = maze_boards(1, 19, seed=0)
    masks = np.ones((2, 1, 361), np.uint8)
    run_kernel("maze", "bf16", boards.inputs, boards.given, 1, masks)  # still works


def test_invalid_batch_raises():
    m = build("maze", seed=0, device=DEV)
    eng = m.engine()
    with pytest.raises(L.NcaError):
        eng.new_state(0, 361)


def test_unclamped_input_state_is_clamped_after_the_first_step():
    """A state loaded from outside the library (not clamped) is stepped with the reference's
    semantics: perception sees the unclamped values, the clamp follows every step
    (src/nca/model.py:503-525, 430-438)."""
    boards = sudoku_boards(4, seed=21)
    K, D = 2, 3
    m = build("sudoku", seed=0, device=DEV, precision="split")
    eng = m.engine()
    B = 4 * K
    b = eng.batch_from_boards(boards.inputs, boards.given, K)
    x = torch.randn((B, 64, 81), generator=torch.Generator().manual_seed(3)).to(DEV) * 0.5
    st = eng.new_state(B, 81)
    eng.load_nchw(st, x)
    masks = (np.random.default_rng(8).random((D, B, 81)) < 0.5).astype(np.uint8)
    eng.run(st, b, D, mode="mask", masks=torch.from_numpy(masks).to(DEV))
    got = eng.store_nchw(st).reshape(B, 64, 9, 9).cpu().numpy()
    eng.check()
    p, _ = oracle_params("sudoku")
    inputs_k = np.repeat(boards.inputs, K, 0)
    given_k = np.repeat(boards.given, K, 0)
    _, g4, clamp = O.init_state(inputs_k, given_k, p, 64)
    ref = x.reshape(B, 64, 9, 9).cpu().numpy()
    for t in range(D):
        ref = O.step(ref, g4, clamp, masks[t].reshape(B, 1, 9, 9).astype(np.float32), p)
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()
