"""`rollout()` of the reference (src/nca/rollout.py:86-305) on the B200 engine.

Same signature and result type as nca.rollout.rollout: boards x K trials are flattened into
one batch (board n -> instances n*K .. n*K+K-1), processed in passes of at most
`max_cells // (K*H*W)` boards, stepped for `depth` steps, scored at the recorded steps and at the
end.  The steps between two observation points (record, prune, end) run as one persistent
kernel launch.

Randomness (RolloutConfig.engine["fire"]):
  "philox" (default) -- in-kernel counter-based Philox4x32-10 keyed by (seed, global instance,
                        cell, step); independent of chunking and of the number of GPUs;
  "torch"            -- the reference's stream: one torch.Generator(seed) on the model's device,
                        `randn` for the initial state of each pass (src/nca/model.py:404) and one
                        `rand((B,1,H,W))` per step (src/nca/model.py:586), consumed in the same
                        order; the kernel applies the drawn masks.  engine["generator"] = "cpu"
                        makes the draws on a CPU generator instead (copied to the device), which
                        replays exactly the stream of a reference run on the CPU.

The reference's options on this path:
  threshold adaptive firing: RolloutConfig.p_low / tau / given_confident (src/nca/model.py:
      566-593), evaluated in the kernel on each cell's confidence;
  test-time noise: RolloutConfig.noise = {"p_t", "p_s", "sigma", "r"} (src/nca/perturb.py:23-40,
      the first r * depth steps): with fire "philox" the instance / cell / Gaussian draws come
      from tagged Philox streams in the kernel; with fire "torch" the reference's own draws
      (fire mask, then noise, per step) are made on the generator and applied by the kernel;
  damage: RolloutConfig.damage_at / damage (src/nca/rollout.py:206-212): the discs are drawn
      on the host from numpy.random.default_rng(seed), the state update is a kernel.

Rules beyond the reference's:
  resident states: RolloutConfig.engine["resident"] (default True) runs the steps between two
      observation points with every instance's state in shared memory where whole instances fit
      (bf16 mode below 64 channels, without noise or confidence rules);
  adaptive firing (continuous):  RolloutConfig.engine["adaptive"] = {"scale": a, "bias": b}
      p_cell = a * (1 - conf_cell) + b with conf_cell = NCA.confidence of the current state;
  niche-capped pruning with refill: RolloutConfig.pruning = {"every": s, "n_cap": c}
      every s steps, per board: group trials by decoded grid, keep the c most confident per
      niche, refill the dropped slots with clones of the kept trials (K stays constant).

The reference's pruning, RolloutConfig.pruning = {"m": m, "n_cap": c}, halves the alive trials
of every board at m - 1 equidistant checkpoints (src/nca/pruning.py:22-65) and compacts the batch
(src/nca/rollout.py:249-275): niches and survivors are computed on the device, the niche orders
are drawn from numpy.random.default_rng(seed) in the reference's order, and the surviving
states are gathered into a smaller state, so the steps after a checkpoint cost less.  A pruned
trial keeps its last values (alive False), and its Philox stream does not change when the batch
is renumbered.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib as L
from ._ops import ops
from .engine import B200Engine
from .perturb import circular_masks, sample_noise
from .tasks import Boards, Task


# With engine["fire"] == "torch", the longest launch (steps) whose draws are made at once.
TORCH_STEP_CHUNK = 64


@dataclass
class RolloutConfig:
    """Fields of nca.rollout.RolloutConfig (src/nca/rollout.py:30-47)."""

    depth: int
    k: int = 1
    fire_rate: float | None = None
    p_low: float | None = None
    tau: float | None = None
    given_confident: bool = True
    noise: dict | None = None
    damage_at: int | None = None
    damage: dict = field(default_factory=lambda: {"n": 1, "r_min": 0.1, "r_max": 0.4})
    pruning: dict | None = None
    record_every: int = 0
    record_boards: int = 0
    max_cells: int = 2_000_000
    amp: bool = False
    local_clock: bool = True
    engine: dict | None = None


@dataclass
class RolloutResult:
    """Same fields as nca.rollout.RolloutResult (src/nca/rollout.py:50-67)."""

    pred: np.ndarray
    conf: np.ndarray
    alive: np.ndarray
    cell_updates: np.ndarray
    steps: np.ndarray
    trace_exact: np.ndarray | None
    trace_cell_acc: np.ndarray | None
    trace_conf: np.ndarray | None
    trace_updates: np.ndarray | None
    boards_trace: np.ndarray | None
    damage_masks: np.ndarray | None

    @property
    def n_boards(self) -> int:
        return self.pred.shape[0]


def _engine_for(model, opts: dict) -> B200Engine:
    precision = opts.get("precision", getattr(model, "precision", "bf16"))
    eng = getattr(model, "_engine", None)
    if isinstance(eng, B200Engine) and eng.precision == precision:
        return eng
    eng = B200Engine(model, precision=precision)
    try:
        model._engine = eng
    except AttributeError:
        pass
    return eng


def _check_config(rc) -> None:
    if (getattr(rc, "p_low", None) is None) != (getattr(rc, "tau", None) is None):
        raise ValueError("threshold adaptive firing needs both p_low and tau")
    if getattr(rc, "p_low", None) is not None and (getattr(rc, "engine", None) or {}).get("adaptive"):
        raise ValueError("choose one adaptive rule: p_low/tau or engine['adaptive']")
    nz = getattr(rc, "noise", None)
    if nz is not None and not all(k in nz for k in ("p_t", "p_s", "sigma")):
        raise ValueError("noise needs p_t, p_s and sigma (src/nca/perturb.py:23-40)")
    pr = getattr(rc, "pruning", None)
    if pr is not None and "every" not in pr and "m" not in pr:
        raise ValueError("pruning needs 'm' (halving at m - 1 checkpoints, src/nca/pruning.py) or "
                         "'every' (niche-capped pruning with refill)")


def _prune_steps(rc) -> tuple[str | None, set[int], int]:
    """(mode, steps after which to prune, n_cap)."""
    pr = rc.pruning
    if not pr:
        return None, set(), 0
    if "m" in pr:  # the reference's checkpoints (src/nca/rollout.py:154-158)
        m = int(pr["m"])
        dt = rc.depth // m
        return "halving", {i * dt for i in range(1, m)}, int(pr.get("n_cap", 3))
    every = int(pr["every"])
    return "refill", set(range(every, rc.depth, every)), int(pr.get("n_cap", 2))


def rollout(model, task: Task, boards: Boards, rc, seed: int = 0, task_ids=None,
            progress: bool = False, board_offset: int = 0) -> RolloutResult:
    """Run every board K times for rc.depth steps on the B200 engine (see module docstring).
    `board_offset` is the global index of boards[0] (multi-GPU shards keep the Philox stream of
    a single-GPU run)."""
    _check_config(rc)
    opts = dict(getattr(rc, "engine", None) or {})
    eng = _engine_for(model, opts)
    cfg = eng.cfg
    dev = eng.device
    fire = opts.get("fire", "philox")
    if fire not in ("philox", "torch"):
        raise ValueError("engine['fire'] must be 'philox' or 'torch'")
    adaptive = opts.get("adaptive")
    # states resident in shared memory between observation points where whole instances fit
    resident = bool(opts.get("resident", True))
    thr = (float(rc.p_low), float(rc.tau), bool(rc.given_confident)) if rc.p_low is not None else None
    p_fire = cfg.fire_rate if rc.fire_rate is None else rc.fire_rate
    noise = rc.noise
    noise_until = int(math.ceil(float(noise.get("r", 1.0)) * rc.depth)) if noise is not None else 0
    damage_at = rc.damage_at
    N = len(boards)
    H, W = boards.shape
    HW = H * W
    K = rc.k
    per_pass = max(1, rc.max_cells // (K * HW))
    gen_where = opts.get("generator", "device")
    if gen_where not in ("device", "cpu"):
        raise ValueError("engine['generator'] must be 'device' or 'cpu'")
    gdev = dev if gen_where == "device" else torch.device("cpu")
    gen = None
    if fire == "torch":
        gen = torch.Generator(device=gdev)
        gen.manual_seed(seed)
    rng = np.random.default_rng(seed)  # host draws: pruning orders (src/nca/rollout.py:103)

    record = rc.record_every > 0
    steps = list(range(rc.record_every, rc.depth + 1, rc.record_every)) if record else []
    if record and (not steps or steps[-1] != rc.depth):
        steps.append(rc.depth)
    T = len(steps)
    prune_mode, prune_steps, n_cap = _prune_steps(rc)

    out_pred = np.zeros((N, K, H, W), dtype=np.int64)
    out_conf = np.zeros((N, K), dtype=np.float32)
    out_alive = np.ones((N, K), dtype=bool)
    out_upd = np.zeros((N, K), dtype=np.float64)
    tr_exact = np.zeros((N, K, T), dtype=bool) if record else None
    tr_cell = np.zeros((N, K, T), dtype=np.float32) if record else None
    tr_conf = np.zeros((N, K, T), dtype=np.float32) if record else None
    tr_upd = np.zeros((N, K, T), dtype=np.float64) if record else None
    boards_trace = np.zeros((rc.record_boards, T, H, W), dtype=np.int64) if rc.record_boards else None
    damage_masks = np.zeros((N, H, W), dtype=bool) if damage_at is not None else None
    boundaries = sorted({rc.depth, *steps, *prune_steps}
                        | ({damage_at} if damage_at is not None and 0 < damage_at < rc.depth else set()))

    for start in range(0, N, per_pass):
        sub = boards.subset(np.arange(start, min(N, start + per_pass)))
        n = len(sub)
        B = n * K
        batch = eng.batch_from_boards(sub.inputs, sub.given, K, inst_offset=(board_offset + start) * K)
        st = eng.new_state(B, HW)
        if fire == "torch" or cfg.sigma_init != 0:
            g0 = gen
            if g0 is None:
                g0 = torch.Generator(device=gdev)
                g0.manual_seed(seed + start)
            x0 = (torch.randn((B, cfg.channels, H, W), generator=g0, device=gdev) * cfg.sigma_init).to(dev)
            eng.load_nchw(st, x0)
            # clamp the given cells: a step where no cell fires
            zero = torch.zeros((1, B, HW), dtype=torch.uint8, device=dev)
            eng.run(st, batch, 1, mode="mask", masks=zero)
        else:
            eng.init_state(st, batch)
        targets = torch.from_numpy(sub.targets).to(dev)
        updates = torch.zeros(B, dtype=torch.int32, device=dev)
        # Compaction (halving): row r of the live batch is (board, trial) idx[r] of this pass.
        idx = torch.arange(B, device=dev)
        # results of the pass by (board, trial), kept on the device until the pass ends
        r_pred = torch.zeros((B, HW), dtype=torch.uint8, device=dev)
        r_conf = torch.zeros(B, dtype=torch.float32, device=dev)
        r_upd = torch.zeros(B, dtype=torch.float64, device=dev)
        r_alive = torch.ones(B, dtype=torch.bool, device=dev)
        if record:
            t_exact = torch.zeros((B, T), dtype=torch.bool, device=dev)
            t_cell = torch.zeros((B, T), dtype=torch.float32, device=dev)
            t_conf = torch.zeros((B, T), dtype=torch.float32, device=dev)
            t_upd = torch.zeros((B, T), dtype=torch.float64, device=dev)
        t = 0
        t_rec = 0
        def damage(t_now: int) -> None:
            dmg = rc.damage
            masks = circular_masks(n, H, W, int(dmg["n"]), float(dmg["r_min"]), float(dmg["r_max"]),
                                   rng, geometry=dmg.get("geometry", "ours"))
            damage_masks[start : start + n] = masks
            eng.damage(st, batch, torch.from_numpy(masks.reshape(n, HW)).to(dev))

        if damage_at == 0:
            damage(0)
        rule = "adaptive" if adaptive is not None else ("threshold" if thr is not None else None)
        for bnd in boundaries:
            n_steps = bnd - t
            Bc = int(idx.numel())
            kw = dict(seed=seed, updates=updates, p_fire=p_fire, resident=resident)
            if adaptive is not None:
                kw["adaptive"] = (float(adaptive.get("scale", 0.9)), float(adaptive.get("bias", 0.1)))
            if thr is not None:
                kw["threshold"] = thr
            if fire == "torch":
                # the reference's stream: per step a fire draw, then (inside the noise window)
                # the noise draws; the kernel applies them
                per_step = noise is not None and t < noise_until
                # launches of at most TORCH_STEP_CHUNK steps, so that a long segment does not hold
                # all of its draws at once; the draws stay in the reference's order
                chunks = ([(t + i, 1) for i in range(n_steps)] if per_step else
                          [(t0, min(TORCH_STEP_CHUNK, bnd - t0)) for t0 in range(t, bnd, TORCH_STEP_CHUNK)])
                for t0, ns in chunks:
                    u = torch.stack([torch.rand((Bc, 1, H, W), generator=gen, device=gdev).reshape(Bc, HW)
                                     for _ in range(ns)]).to(dev)
                    nz = None
                    if per_step and t0 < noise_until:
                        tn = sample_noise(Bc, cfg.channels, H, W, noise["p_t"], noise["p_s"],
                                          noise["sigma"], gen, gdev)
                        nz = None if tn is None else {"tensor": tn.reshape(Bc, cfg.channels, HW).to(dev)}
                    if rule is None:
                        eng.run(st, batch, ns, mode="mask", masks=(u < p_fire).to(torch.uint8),
                                step0=t0, noise=nz, **kw)
                    else:
                        eng.run(st, batch, ns, mode=rule + "_uniform", uniforms=u, step0=t0, noise=nz, **kw)
            else:
                nz = None
                if noise is not None and t < noise_until:
                    nz = {"p_t": noise["p_t"], "p_s": noise["p_s"], "sigma": noise["sigma"],
                          "until": noise_until}
                eng.run(st, batch, n_steps, mode=rule or "philox", step0=t, noise=nz, **kw)
            t = bnd
            if t in prune_steps and prune_mode == "refill":
                r = eng.readout(st, batch)
                src, _ = eng.prune_refill(st, r["pred"], r["board_conf"], n, K, n_cap)
                updates = updates.index_select(0, src.long())  # a clone continues its source's count
            elif t in prune_steps:
                # halving with compaction (src/nca/rollout.py:249-275)
                r = eng.readout(st, batch, targets=targets)
                per_board = np.bincount(torch.div(idx, K, rounding_mode="floor").cpu().numpy(),
                                        minlength=n)
                keep = eng.halving(r["pred"], r["board_conf"], per_board, n_cap, rng).bool()
                drop = ~keep
                if bool(drop.any()):
                    rows = idx[drop]
                    r_pred[rows] = r["pred"][drop]
                    r_conf[rows] = r["board_conf"][drop]
                    r_upd[rows] = updates[drop].double()
                    r_alive[rows] = False
                    if record and t_rec < T:
                        # a trajectory that leaves keeps its last values for the remaining records
                        t_exact[rows, t_rec:] = r["exact"][drop].bool()[:, None]
                        t_cell[rows, t_rec:] = r["cell_acc"][drop][:, None]
                        t_conf[rows, t_rec:] = r["board_conf"][drop][:, None]
                        t_upd[rows, t_rec:] = updates[drop].double()[:, None]
                    sel = keep.nonzero().squeeze(1)
                    st = eng.gather(st, sel)
                    batch = eng.compacted(batch, sel)
                    updates = updates[sel]
                    idx = idx[sel]
            if record and T and t_rec < T and t == steps[t_rec]:
                r = eng.readout(st, batch, targets=targets)
                t_exact[idx, t_rec] = r["exact"].bool()
                t_cell[idx, t_rec] = r["cell_acc"]
                t_conf[idx, t_rec] = r["board_conf"]
                t_upd[idx, t_rec] = updates.double()
                if boards_trace is not None and start < rc.record_boards:
                    # the first trial of the first boards (its last decoded grid if it was pruned)
                    r_pred[idx] = r["pred"]
                    nb = min(n, rc.record_boards - start)
                    dec = r_pred.reshape(n, K, H, W)[:nb, 0].long().cpu().numpy()
                    boards_trace[start : start + nb, t_rec] = dec
                t_rec += 1
            if damage_at is not None and t == damage_at and 0 < t < rc.depth:
                damage(t)
        r = eng.readout(st, batch)
        eng.check()
        r_pred[idx] = r["pred"]
        r_conf[idx] = r["board_conf"]
        r_upd[idx] = updates.double()
        # the decoded tokens cross as bytes and widen to int64 in the host array's own write
        out_pred[start : start + n] = r_pred.reshape(n, K, H, W).cpu().numpy()
        out_conf[start : start + n] = r_conf.reshape(n, K).cpu().numpy()
        out_upd[start : start + n] = r_upd.reshape(n, K).cpu().numpy()
        out_alive[start : start + n] = r_alive.reshape(n, K).cpu().numpy()
        if record:
            tr_exact[start : start + n] = t_exact.reshape(n, K, T).cpu().numpy()
            tr_cell[start : start + n] = t_cell.reshape(n, K, T).cpu().numpy()
            tr_conf[start : start + n] = t_conf.reshape(n, K, T).cpu().numpy()
            tr_upd[start : start + n] = t_upd.reshape(n, K, T).cpu().numpy()

    return RolloutResult(out_pred, out_conf, out_alive, out_upd, np.array(steps), tr_exact,
                         tr_cell, tr_conf, tr_upd, boards_trace, damage_masks)


def decode_boards(model, task: Task, x: torch.Tensor, given: torch.Tensor, inputs: torch.Tensor):
    """src/nca/rollout.py:74-82."""
    dec = model.decode(x)
    return torch.where(given.to(dec.device), inputs.to(dec.device), dec) if task.fill_given else dec


def score_candidates(task: Task, res: RolloutResult, boards: Boards) -> dict[str, np.ndarray]:
    """Task metrics for every (board, trial) (src/nca/rollout.py:309-314)."""
    N, K, H, W = res.pred.shape
    m = task.metrics(res.pred.reshape(N * K, H, W), boards.repeat(K))
    return {k: np.asarray(v).reshape(N, K) for k, v in m.items()}


def select_best(conf: np.ndarray, alive: np.ndarray, k: int, device=None) -> np.ndarray:
    """Per board, the first index of the largest confidence among alive trials k' < k, computed
    by the library's selection kernel (the argmax of src/nca/rollout.py:331-332)."""
    N, K = conf.shape
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    c = torch.from_numpy(np.ascontiguousarray(conf, dtype=np.float32)).to(dev)
    a = torch.from_numpy(np.ascontiguousarray(alive, dtype=np.uint8)).to(dev)
    idx = torch.empty(N, dtype=torch.int32, device=dev)
    best = torch.empty(N, dtype=torch.float32, device=dev)
    ops().select(c, a, N, K, int(min(k, K)), idx, best, None, 0, None)
    return idx.cpu().numpy().astype(np.int64)


def conf_at_k(metric: np.ndarray, conf: np.ndarray, alive: np.ndarray, ks: list[int],
              weights: np.ndarray | None = None, device=None) -> dict[int, float]:
    """Conf@k for several k (src/nca/rollout.py:317-334): per board the alive trial of highest
    confidence among the first k, then the (weighted) mean of its metric."""
    N, K = metric.shape
    out = {}
    for k in ks:
        k = min(k, K)
        best = select_best(conf, alive, k, device)
        out[k] = float(np.average(metric[np.arange(N), best], weights=weights))
    return out


def pass_at_k(metric: np.ndarray, alive: np.ndarray, ks: list[int],
              weights: np.ndarray | None = None) -> dict[int, float]:
    """Pass@k (src/nca/rollout.py:337-350): any of the first k alive trials correct."""
    N, K = metric.shape
    return {
        min(k, K): float(np.average((metric[:, : min(k, K)] & alive[:, : min(k, K)]).any(axis=1),
                                    weights=weights))
        for k in ks
    }
