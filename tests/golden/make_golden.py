"""Generate tests/golden/golden.npz from the live reference (JorisViaudQuantAI/NCAs).

Run in a container where the reference is importable (it is not on the GPU box):

    PYTHONPATH=/path/to/reference/src python tests/golden/make_golden.py /path/to/reference
    PYTHONPATH=/path/to/reference/src python tests/golden/make_golden.py /path/to/reference long

Every array in the file is produced by the reference's own code: nca.model.NCA (built through
nca.model.build_model with the benchmark overrides and the benchmark's synthetic weights loaded
into it), nca.rollout.conf_at_k / pass_at_k, nca.pruning.niche_capped_pruning and the maze /
sudoku generators of nca.tasks.  The tests compare the oracle and the CUDA kernels against it.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[2]
if len(sys.argv) < 2:
    raise SystemExit("usage: python tests/golden/make_golden.py <reference checkout>")
REF = Path(sys.argv[1])
sys.path.insert(0, str(REF / "src"))
sys.path.insert(0, str(REPO))

from nca.model import build_model  # noqa: E402  (reference)
from nca.pruning import niche_capped_pruning  # noqa: E402
from nca.rollout import conf_at_k, pass_at_k  # noqa: E402
from nca.tasks.maze import generate_hard_maze, generate_perfect_maze  # noqa: E402
from nca.tasks.sudoku import sudoku_symmetry  # noqa: E402

from ncas_b200.configs import model_config, synthetic_params  # noqa: E402

torch.set_num_threads(4)
OUT = Path(__file__).resolve().parent / "golden.npz"
G: dict[str, np.ndarray] = {}


def ref_model(task: str, seed: int):
    cfg = model_config(task)
    d = {k: v for k, v in cfg.to_dict().items()}
    m = build_model(None, **d)
    with torch.no_grad():
        for name, v in synthetic_params(cfg, seed).items():
            m.get_parameter(name).copy_(torch.from_numpy(v))
    m.eval()
    return m


def second_endpoint_goal(inp: np.ndarray) -> np.ndarray:
    """D8: the reference's maze-OOD endpoints are both token 3; the one second in row-major
    order becomes the goal (token 4), as nca.tasks.maze._second_endpoint_as_goal does."""
    t = inp.astype(np.int64).copy()
    ends = np.argwhere(t == 3)
    t[tuple(ends[1])] = 4
    return t


def run_steps(m, inputs, given, K, masks, record=(1,)):
    inp = torch.from_numpy(np.repeat(inputs, K, 0))
    gv = torch.from_numpy(np.repeat(given, K, 0))
    x, g4, clamp = m.init_state(inp, gv)
    rec = {}
    with torch.no_grad():
        for t in range(masks.shape[0]):
            fm = torch.from_numpy(masks[t].reshape(x.shape[0], 1, *x.shape[2:]).astype(np.float32))
            x = m.step(x, g4, clamp, fm)
            if t + 1 in record:
                rec[t + 1] = x.numpy().copy()
        dec = torch.where(gv, inp, m.decode(x))
        return rec, x.numpy(), dec.numpy(), m.confidence(x).numpy(), m.board_confidence(x).numpy()


def main() -> None:
    # ---- maze boards: perfect 19x19 (cfg0 shape), reference generator
    rng = np.random.default_rng(7)
    mz = [generate_perfect_maze(19, rng) for _ in range(4)]
    maze_inputs = np.stack([second_endpoint_goal(i) for i, _ in mz])
    maze_targets = np.stack([second_endpoint_goal(t) for _, t in mz])
    G["maze_inputs"], G["maze_targets"] = maze_inputs.astype(np.uint8), maze_targets.astype(np.uint8)
    rng = np.random.default_rng(8)
    hard = [generate_hard_maze(30, rng, min_path_len=60, extra_openings=0.10) for _ in range(2)]
    G["hard_inputs"] = np.stack([h[0] for h in hard]).astype(np.uint8)

    # ---- maze rollout: 4 boards, K=1, 64 steps, seeded external masks
    m = ref_model("maze", 0)
    maze_given = maze_inputs != 0
    masks = (np.random.default_rng(11).random((64, 4, 19 * 19)) < 0.5).astype(np.uint8)
    rec, x64, dec, cconf, bconf = run_steps(m, maze_inputs, maze_given, 1, masks, record=(1,))
    G.update(maze_masks=masks, maze_x1=rec[1], maze_x64=x64, maze_dec64=dec.astype(np.uint8),
             maze_cconf64=cconf, maze_bconf64=bconf)

    # ---- sudoku: 4 boards, K=2, 64 steps
    rng = np.random.default_rng(21)
    syms = [sudoku_symmetry(rng) for _ in range(3)]
    G["sym_rows"] = np.stack([s[0] for s in syms])
    G["sym_cols"] = np.stack([s[1] for s in syms])
    G["sym_tr"] = np.array([s[2] for s in syms])
    G["sym_digits"] = np.stack([s[3] for s in syms])
    from ncas_b200.tasks import sudoku_boards

    sb = sudoku_boards(4, seed=5)
    G["sudoku_inputs"], G["sudoku_given"] = sb.inputs.astype(np.uint8), sb.given
    G["sudoku_targets"] = sb.targets.astype(np.uint8)
    m = ref_model("sudoku", 0)
    masks = (np.random.default_rng(12).random((64, 8, 81)) < 0.5).astype(np.uint8)
    rec, x64, dec, cconf, bconf = run_steps(m, sb.inputs, sb.given, 2, masks, record=(1,))
    G.update(sudoku_masks=masks, sudoku_x1=rec[1], sudoku_x64=x64, sudoku_dec64=dec.astype(np.uint8),
             sudoku_cconf64=cconf, sudoku_bconf64=bconf)

    # ---- adaptive (continuous rule on the reference's confidence), 16 steps
    inp = torch.from_numpy(np.repeat(sb.inputs, 2, 0))
    gv = torch.from_numpy(np.repeat(sb.given, 2, 0))
    x, g4, clamp = m.init_state(inp, gv)
    u = np.random.default_rng(13).random((16, 8, 81)).astype(np.float32)
    fired = np.zeros(8, np.int64)
    with torch.no_grad():
        for t in range(16):
            conf = m.confidence(x)[:, None]
            prob = 0.9 * (1 - conf) + 0.1
            fm = (torch.from_numpy(u[t].reshape(8, 1, 9, 9)) < prob).float()
            fired += fm.reshape(8, -1).sum(1).long().numpy()
            x = m.step(x, g4, clamp, fm)
    G.update(adapt_u=u, adapt_x16=x.numpy(), adapt_fired=fired,
             adapt_dec16=torch.where(gv, inp, m.decode(x)).numpy().astype(np.uint8))

    # ---- conf@K / pass@K on random inputs
    r = np.random.default_rng(31)
    metric = r.random((20, 8)) < 0.4
    conf = r.random((20, 8)).astype(np.float32)
    conf[3, 2] = conf[3, 5]  # a tie: the first index must win
    alive = r.random((20, 8)) < 0.8
    ks = [1, 2, 4, 8]
    ck, pk = conf_at_k(metric, conf, alive, ks), pass_at_k(metric, alive, ks)
    G.update(sel_metric=metric, sel_conf=conf, sel_alive=alive,
             sel_confk=np.array([ck[k] for k in ks]), sel_passk=np.array([pk[k] for k in ks]))

    # ---- niche-capped pruning (reference halving rule) with its rng
    r = np.random.default_rng(41)
    dec = r.integers(0, 3, size=(6, 8, 2, 2))
    dec[:, :4] = dec[:, :1]  # duplicates: trials 0..3 share a niche
    pconf = r.random((6, 8)).astype(np.float32)
    palive = np.ones((6, 8), dtype=bool)
    palive[5, 6:] = False
    new = niche_capped_pruning(torch.from_numpy(dec), torch.from_numpy(pconf), torch.from_numpy(palive),
                               2, np.random.default_rng(42))
    G.update(prune_dec=dec, prune_conf=pconf, prune_alive=palive, prune_new=new.numpy())

    # ---- perturbations (damage discs, noise draws) and the threshold firing rule
    from nca.perturb import circular_masks as ref_circular_masks  # noqa: E402
    from nca.perturb import sample_noise as ref_sample_noise  # noqa: E402

    G["dmg_ours"] = ref_circular_masks(4, 15, 13, 2, 0.1, 0.4, np.random.default_rng(21))
    G["dmg_official"] = ref_circular_masks(3, 9, 9, 1, 0.2, 0.5, np.random.default_rng(22),
                                           geometry="official")
    nz = ref_sample_noise(torch.zeros((6, 8, 5, 5)), 0.6, 0.5, 0.05, torch.Generator().manual_seed(7))
    G["noise_draw"] = nz.numpy()
    g4_np = gv.numpy()[:, None]
    fm_g = m.sample_fire_mask(x, 0.5, 0.1, 0.12, torch.Generator().manual_seed(3), g4)
    fm_n = m.sample_fire_mask(x, 0.5, 0.1, 0.12, torch.Generator().manual_seed(3), None)
    u_thr = torch.rand((8, 1, 9, 9), generator=torch.Generator().manual_seed(3))
    G.update(thr_x=x.numpy(), thr_given=g4_np, thr_u=u_thr.numpy(), thr_mask_given=fm_g.numpy(),
             thr_mask=fm_n.numpy())

    np.savez_compressed(OUT, **G)
    print(f"wrote {OUT} ({OUT.stat().st_size / 1e3:.0f} kB, {len(G)} arrays)")
    presets()


def presets() -> None:
    """The reference's trained maze presets (runs/engine/*_opt/seed0/final.pt) stepped by the
    reference's own model: their weights and buffers, seeded boards, initial states, external
    masks and the states after 1 and 12 steps, decoded boards and confidences."""
    import json

    from nca.tasks.maze import generate_hard_maze as ghm  # noqa: E402
    from nca.tasks.maze import generate_perfect_maze as gpm  # noqa: E402
    from nca.train import load_model  # noqa: E402

    P: dict[str, np.ndarray] = {}
    cases = {
        "maze_ood": lambda r: gpm(19, r)[:2],
        "maze_hard": lambda r: ghm(30, r, min_path_len=60, extra_openings=0.10)[:2],
    }
    for i, (name, gen) in enumerate(cases.items()):
        m, _ = load_model(REF / "runs" / "engine" / f"{name}_opt" / "seed0" / "final.pt", device="cpu")
        ck = torch.load(REF / "runs" / "engine" / f"{name}_opt" / "seed0" / "final.pt",
                        map_location="cpu", weights_only=False)
        for k, v in ck["model"].items():
            P[f"{name}__w__{k}"] = v.float().numpy()
        P[f"{name}__config"] = np.array(json.dumps(ck["model_config"]))
        r = np.random.default_rng(51 + i)
        pairs = [gen(r) for _ in range(3)]
        inputs = np.stack([a for a, _ in pairs]).astype(np.int64)
        P[f"{name}__targets"] = np.stack([b for _, b in pairs]).astype(np.uint8)
        given = inputs != 0
        inp = torch.from_numpy(inputs)
        gv = torch.from_numpy(given)
        with torch.no_grad():
            x, g4, clamp = m.init_state(inp, gv, None, torch.Generator().manual_seed(3))
            B, _, H, W = x.shape
            masks = (np.random.default_rng(61 + i).random((100, B, H * W)) < 0.8).astype(np.uint8)
            P[f"{name}__x0"] = x.numpy().copy()
            for t in range(100):
                fm = torch.from_numpy(masks[t].reshape(B, 1, H, W).astype(np.float32))
                x = m.step(x, g4, clamp, fm)
                if t == 0:
                    P[f"{name}__x1"] = x.numpy().copy()
                if t == 11:
                    P[f"{name}__x12"] = x.numpy().copy()
                    P[f"{name}__dec12"] = torch.where(gv, inp, m.decode(x)).numpy().astype(np.uint8)
                    P[f"{name}__cconf12"] = m.confidence(x).numpy()
                    P[f"{name}__bconf12"] = m.board_confidence(x).numpy()
            # a 100-step rollout (the presets' evaluation depth for maze_ood): decoded boards
            P[f"{name}__dec100"] = torch.where(gv, inp, m.decode(x)).numpy().astype(np.uint8)
            P[f"{name}__bconf100"] = m.board_confidence(x).numpy()
        P[f"{name}__inputs"] = inputs.astype(np.uint8)
        P[f"{name}__given"] = given
        P[f"{name}__masks"] = masks
    out = OUT.parent / "presets.npz"
    np.savez_compressed(out, **P)
    print(f"wrote {out} ({out.stat().st_size / 1e3:.0f} kB, {len(P)} arrays)")


def long_rollout() -> None:
    """A long rollout for the task-level agreement check: the reference's trained maze_ood preset
    run by the reference's own rollout() on 100 seeded 59x59 perfect mazes (a 29x29-cell maze)
    for D = 2000 steps, the depth the reference's Table 1 uses at that size
    (scripts/eval_maze_scaling.py:26, TABLE1 = {13: 300, 59: 2000, 201: 13000}).  K = 1, the
    rollout's own torch.Generator(seed) on the CPU (randn initial state, one rand mask per step),
    so a GPU run that replays the same draws sees the same fire masks.  Stored: the boards, the
    per-board exact flags, the decoded final boards, the board confidences and update counts."""
    from nca.rollout import RolloutConfig, rollout, score_candidates  # noqa: E402
    from nca.tasks.base import Boards as RefBoards  # noqa: E402
    from nca.tasks.maze import MazeOOD  # noqa: E402
    from nca.train import load_model  # noqa: E402

    torch.set_num_threads(8)
    m, _ = load_model(REF / "runs" / "engine" / "maze_ood_opt" / "seed0" / "final.pt", device="cpu")
    rng = np.random.default_rng(LONG_BOARD_SEED)
    pairs = [generate_perfect_maze(LONG_SIZE, rng) for _ in range(LONG_N)]
    inputs = np.stack([a for a, _ in pairs]).astype(np.int64)
    targets = np.stack([b for _, b in pairs]).astype(np.int64)
    boards = RefBoards(inputs, targets, inputs != 0)
    task = MazeOOD()
    rc = RolloutConfig(depth=LONG_DEPTH, k=1, record_every=LONG_DEPTH // 4)
    res = rollout(m, task, boards, rc, seed=LONG_ROLLOUT_SEED)
    met = score_candidates(task, res, boards)
    P = dict(inputs=inputs.astype(np.uint8), targets=targets.astype(np.uint8),
             exact=np.asarray(met["exact"]).reshape(LONG_N).astype(bool),
             pred=res.pred[:, 0].astype(np.uint8), conf=res.conf[:, 0],
             updates=res.cell_updates[:, 0], trace_exact=res.trace_exact[:, 0],
             steps=res.steps, depth=np.array(LONG_DEPTH), rollout_seed=np.array(LONG_ROLLOUT_SEED),
             board_seed=np.array(LONG_BOARD_SEED))
    out = OUT.parent / "long_rollout.npz"
    np.savez_compressed(out, **P)
    print(f"wrote {out} ({out.stat().st_size / 1e3:.0f} kB); reference exact rate "
          f"{P['exact'].mean():.3f}, trace {res.trace_exact[:, 0].mean(0)}")


LONG_N, LONG_SIZE, LONG_DEPTH = 100, 59, 2000
LONG_BOARD_SEED, LONG_ROLLOUT_SEED = 71, 5

if __name__ == "__main__":
    if len(sys.argv) > 2 and sys.argv[2] == "long":
        long_rollout()
    else:
        main()
