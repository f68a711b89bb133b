"""Task-level agreement of a long rollout with the reference.

The reference's trained maze_ood preset was run by the reference's own rollout() on 100 seeded
59x59 mazes for D = 2000 steps (the depth of the reference's Table 1 at that size,
scripts/eval_maze_scaling.py:26), on the CPU with its torch.Generator stream, and its per-board
exact-match flags were recorded (tests/golden/long_rollout.npz, made by
tests/golden/make_golden.py).  The library's rollout() runs the same boards with the same
weights:

* replaying the reference's draws (engine fire "torch" on a CPU generator: the same initial
  state and the same 2000 fire masks), in both precisions: the exact-match rate must be within
  1 point of the reference's, and the per-board flags must agree for at least 99 of 100 boards;
* with the in-kernel Philox stream (other random masks, so only the rate is comparable): within
  1 point.
"""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from ncas_b200.model import NCA, NCAConfig
from ncas_b200.rollout import RolloutConfig, rollout
from ncas_b200.tasks import Boards, MazeOODTask

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
GOLD = Path(__file__).resolve().parent / "golden"


def preset_model(precision: str):
    g = np.load(GOLD / "presets.npz")
    cfg = NCAConfig.from_dict(json.loads(str(g["maze_ood__config"])))
    m = NCA(cfg, precision=precision)
    m.load_state_dict({k.split("__w__")[1]: torch.from_numpy(g[k]) for k in g.files
                       if k.startswith("maze_ood__w__")})
    return m.to(DEV)


def exact_flags(engine: dict, precision: str):
    L = np.load(GOLD / "long_rollout.npz")
    inputs = L["inputs"].astype(np.int64)
    boards = Boards(inputs, L["targets"].astype(np.int64), inputs != 0)
    rc = RolloutConfig(depth=int(L["depth"]), k=1, engine={"precision": precision, **engine})
    task = MazeOODTask()
    res = rollout(preset_model(precision), task, boards, rc, seed=int(L["rollout_seed"]))
    got = np.asarray(task.metrics(res.pred[:, 0], boards)["exact"]).astype(bool)
    return got, L["exact"]


@pytest.mark.parametrize("precision", ["split", "bf16"])
def test_long_rollout_replaying_reference_draws_agrees(precision):
    got, ref = exact_flags({"fire": "torch", "generator": "cpu"}, precision)
    assert abs(got.mean() - ref.mean()) <= 0.01, (got.mean(), ref.mean())
    assert (got == ref).sum() >= len(ref) - 1, np.flatnonzero(got != ref)


def test_long_rollout_philox_stream_rate_agrees():
    got, ref = exact_flags({"fire": "philox"}, "bf16")
    assert abs(got.mean() - ref.mean()) <= 0.01, (got.mean(), ref.mean())
