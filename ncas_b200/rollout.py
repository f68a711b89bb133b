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
                        order; the kernel applies the drawn masks.

Rules beyond the reference's uniform firing:
  adaptive firing (continuous):  RolloutConfig.engine["adaptive"] = {"scale": a, "bias": b}
      p_cell = a * (1 - conf_cell) + b with conf_cell = NCA.confidence of the current state;
  niche-capped pruning with refill: RolloutConfig.pruning = {"every": s, "n_cap": c}
      every s steps, per board: group trials by decoded grid, keep the c most confident per
      niche, refill the dropped slots with clones of the kept trials (K stays constant).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib as L
from .engine import B200Engine
from .tasks import Boards, Task


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
    if getattr(rc, "p_low", None) is not None or getattr(rc, "tau", None) is not None:
        raise ValueError("threshold adaptive firing (p_low/tau) is not implemented by the b200 "
                         "backend; use engine['adaptive'] for the continuous rule")
    if getattr(rc, "noise", None) is not None:
        raise ValueError("test-time noise is not implemented by the b200 backend")
    if getattr(rc, "damage_at", None) is not None:
        raise ValueError("damage events are not implemented by the b200 backend")
    pr = getattr(rc, "pruning", None)
    if pr is not None and "every" not in pr:
        raise ValueError("the b200 backend implements niche-capped pruning with refill "
                         "(pruning={'every': s, 'n_cap': c})")


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
    p_fire = cfg.fire_rate if rc.fire_rate is None else rc.fire_rate
    N = len(boards)
    H, W = boards.shape
    HW = H * W
    K = rc.k
    per_pass = max(1, rc.max_cells // (K * HW))
    gen = None
    if fire == "torch":
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)

    record = rc.record_every > 0
    steps = list(range(rc.record_every, rc.depth + 1, rc.record_every)) if record else []
    if record and (not steps or steps[-1] != rc.depth):
        steps.append(rc.depth)
    T = len(steps)
    prune_every = int(rc.pruning["every"]) if rc.pruning else 0
    n_cap = int(rc.pruning.get("n_cap", 2)) if rc.pruning else 0
    prune_steps = set(range(prune_every, rc.depth, prune_every)) if prune_every else set()

    out_pred = np.zeros((N, K, H, W), dtype=np.int64)
    out_conf = np.zeros((N, K), dtype=np.float32)
    out_alive = np.ones((N, K), dtype=bool)
    out_upd = np.zeros((N, K), dtype=np.float64)
    tr = {k: [] for k in ("exact", "cell", "conf", "upd")}
    boards_trace = np.zeros((rc.record_boards, T, H, W), dtype=np.int64) if rc.record_boards else None
    boundaries = sorted({rc.depth, *steps, *prune_steps})

    for start in range(0, N, per_pass):
        sub = boards.subset(np.arange(start, min(N, start + per_pass)))
        n = len(sub)
        B = n * K
        batch = eng.batch_from_boards(sub.inputs, sub.given, K, inst_offset=(board_offset + start) * K)
        st = eng.new_state(B, HW)
        if fire == "torch" or cfg.sigma_init != 0:
            g0 = gen
            if g0 is None:
                g0 = torch.Generator(device=dev)
                g0.manual_seed(seed + start)
            x0 = torch.randn((B, cfg.channels, H, W), generator=g0, device=dev) * cfg.sigma_init
            eng.load_nchw(st, x0)
            # clamp the given cells: a step where no cell fires
            zero = torch.zeros((1, B, HW), dtype=torch.uint8, device=dev)
            eng.run(st, batch, 1, mode="mask", masks=zero)
        else:
            eng.init_state(st, batch)
        targets = torch.from_numpy(sub.targets).to(dev)
        updates = torch.zeros(B, dtype=torch.int32, device=dev)
        p_tr = {k: [] for k in tr}
        t = 0
        t_rec = 0
        for bnd in boundaries:
            n_steps = bnd - t
            kw = dict(seed=seed, step0=t, updates=updates, p_fire=p_fire)
            if adaptive is not None:
                kw["adaptive"] = (float(adaptive.get("scale", 0.9)), float(adaptive.get("bias", 0.1)))
            if fire == "torch":
                u = torch.stack([torch.rand((B, 1, H, W), generator=gen, device=dev).reshape(B, HW)
                                 for _ in range(n_steps)])
                if adaptive is None:
                    eng.run(st, batch, n_steps, mode="mask", masks=(u < p_fire).to(torch.uint8), **kw)
                else:
                    eng.run(st, batch, n_steps, mode="adaptive_uniform", uniforms=u, **kw)
            else:
                eng.run(st, batch, n_steps, mode="adaptive" if adaptive is not None else "philox", **kw)
            t = bnd
            if t in prune_steps:
                r = eng.readout(st, batch)
                src, _ = eng.prune_refill(st, r["pred"], r["board_conf"], n, K, n_cap)
                updates = updates.index_select(0, src.long())  # a clone continues its source's count
            if record and T and t_rec < T and t == steps[t_rec]:
                r = eng.readout(st, batch, targets=targets)
                p_tr["exact"].append(r["exact"].bool())
                p_tr["cell"].append(r["cell_acc"])
                p_tr["conf"].append(r["board_conf"])
                p_tr["upd"].append(updates.double())
                if boards_trace is not None and start < rc.record_boards:
                    nb = min(n, rc.record_boards - start)
                    dec = r["pred"].reshape(n, K, H, W)[:nb, 0].long().cpu().numpy()
                    boards_trace[start : start + nb, t_rec] = dec
                t_rec += 1
        r = eng.readout(st, batch)
        eng.check()
        out_pred[start : start + n] = r["pred"].reshape(n, K, H, W).long().cpu().numpy()
        out_conf[start : start + n] = r["board_conf"].reshape(n, K).cpu().numpy()
        out_upd[start : start + n] = updates.double().reshape(n, K).cpu().numpy()
        for k in tr:
            if p_tr[k]:
                tr[k].append(torch.stack(p_tr[k], dim=1).reshape(n, K, -1).cpu().numpy())

    def cat(k, dtype):
        return np.concatenate(tr[k], axis=0).astype(dtype) if record else None

    return RolloutResult(
        out_pred, out_conf, out_alive, out_upd, np.array(steps),
        cat("exact", bool), cat("cell", np.float32), cat("conf", np.float32), cat("upd", np.float64),
        boards_trace, None,
    )


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
    stream = torch.cuda.current_stream(dev).cuda_stream
    L.check(L.lib().nca_b200_select(c.data_ptr(), a.data_ptr(), N, K, int(min(k, K)), idx.data_ptr(),
                                    best.data_ptr(), None, 0, None, stream), "nca_b200_select")
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
