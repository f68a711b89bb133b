"""The five benchmark configurations: cell-rule configs, synthetic weights and boards.

Each config is a model the reference's NCAConfig can express (nca.model.NCAConfig,
src/nca/model.py:48-137) with:

* perception = 4 fixed 3x3 heads (identity, Sobel-x, Sobel-y, Laplacian) written into
  perceive.weight, zero padding, head-major z[k*C + c];
* MLP 4C -> 4C (ReLU) -> C with both biases, hidden_from_perception=True, expansion=1;
* weights drawn N(0, 0.02) from numpy's default_rng(seed) and rounded to bf16 values (so the fp32
  reference and the bf16 tensor-core path use identical weights), biases 0;
* sigma_init = 0 (zero state), one-hot input embedding, head='mlp' set to the identity on the
  readout slice (decode = argmax of the readout channels, confidence = max softmax).

Maze models: vocab 5 (0 empty, 1 path, 2 wall, 3 start, 4 goal), c_in = 5, readout channels 0-1
(tokens 0, 1).  Sudoku models: vocab 10 (0 empty, 1-9), c_in = 10, readout channels 1-9
(tokens 1..9).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .model import FIXED_TAPS, NCA, NCAConfig
from .tasks import Boards, MazeTask, SudokuTask, maze_boards, sudoku_boards


@dataclass(frozen=True)
class BenchConfig:
    name: str
    task: str            # "maze" | "sudoku"
    n_boards: int
    size: int            # board side (maze) / 9 (sudoku)
    k: int
    depth: int
    p_fire: float = 0.5
    prune_every: int = 0
    n_cap: int = 2
    adaptive: bool = False
    hard: bool = False
    clues: tuple[int, int] = (17, 35)

    @property
    def hw(self) -> int:
        return self.size * self.size

    @property
    def channels(self) -> int:
        return 32 if self.task == "maze" else 64

    @property
    def flop_per_cell_update(self) -> int:
        C = self.channels
        P = 4 * C
        return 2 * (P * P + P * C)

    def bytes_per_cell_update(self, precision: str = "bf16") -> int:
        """Algorithmic HBM bytes of one cell-update of the step kernel.  bf16 mode with C >= 64
        keeps the state as bf16 hi + lo parts: the window reads hi (2C), the epilogue reads lo
        (2C) and writes both (4C) = 8C.  Otherwise the window reads the bf16 mirror (2C; fp32
        in split mode, 4C), the epilogue reads the fp32 state (4C) and writes it (4C) plus the
        mirror (2C in bf16 mode) = 12C."""
        C = self.channels
        if precision == "bf16":
            return 8 * C if C >= 64 else 12 * C
        return 12 * C

    @property
    def cell_updates(self) -> int:
        return self.n_boards * self.k * self.hw * self.depth


CONFIGS = {
    "cfg0": BenchConfig("cfg0", "maze", 64, 19, 1, 64),
    "cfg1": BenchConfig("cfg1", "maze", 1, 201, 1, 13000),
    "cfg2": BenchConfig("cfg2", "sudoku", 1000, 9, 128, 256),
    "cfg3": BenchConfig("cfg3", "maze", 1000, 30, 64, 200, prune_every=20, n_cap=2, hard=True),
    "cfg4": BenchConfig("cfg4", "sudoku", 1000, 9, 512, 2048, adaptive=True, clues=(17, 22)),
}


def model_config(task: str) -> NCAConfig:
    common = dict(
        perception="kernels", heads=4, padding="zero", update="mlp", expansion=1,
        hidden_from_perception=True, sigma_init=0.0, fire_rate=0.5, head="mlp",
        embedding="onehot", zero_init_update=False, wall_token=2,
    )
    if task == "maze":
        return NCAConfig(vocab_size=5, channels=32, c_in=5, c_out=2, output_tokens=(0, 1), **common)
    if task == "sudoku":
        return NCAConfig(vocab_size=10, channels=64, c_in=10, c_out=9, out_offset=1,
                         output_tokens=tuple(range(1, 10)), **common)
    raise ValueError(task)


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16 value (ties to even), returned as fp32."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def synthetic_params(cfg: NCAConfig, seed: int) -> dict[str, np.ndarray]:
    """The benchmark weights as fp32 arrays with the reference's parameter names/shapes."""
    rng = np.random.default_rng(seed)
    C, P = cfg.channels, cfg.heads * cfg.channels
    Hd = cfg.hidden
    w1 = bf16_round(rng.standard_normal((Hd, P)).astype(np.float32) * np.float32(0.02))
    w2 = bf16_round(rng.standard_normal((C, Hd)).astype(np.float32) * np.float32(0.02))
    n_out = len(cfg.output_tokens)
    return {
        "perceive.weight": FIXED_TAPS.reshape(4, 1, 3, 3).copy(),
        "update.fc1.weight": w1.reshape(Hd, P, 1, 1),
        "update.fc1.bias": np.zeros(Hd, np.float32),
        "update.fc2.weight": w2.reshape(C, Hd, 1, 1),
        "update.fc2.bias": np.zeros(C, np.float32),
        "head.weight": np.eye(n_out, cfg.c_out, dtype=np.float32).reshape(n_out, cfg.c_out, 1, 1),
        "head.bias": np.zeros(n_out, np.float32),
    }


def build(task: str, seed: int = 0, device="cuda", precision: str = "bf16") -> NCA:
    """The benchmark model of `task` with its synthetic weights, on `device`."""
    cfg = model_config(task)
    m = NCA(cfg, precision=precision)
    params = synthetic_params(cfg, seed)
    with torch.no_grad():
        for name, v in params.items():
            m.get_parameter(name).copy_(torch.from_numpy(v))
    return m.to(device)


def boards_for(bc: BenchConfig, seed: int = 0, n: int | None = None) -> Boards:
    n = bc.n_boards if n is None else n
    if bc.task == "maze":
        return maze_boards(n, bc.size, seed, hard=bc.hard)
    return sudoku_boards(n, seed, clues=bc.clues)


def task_for(bc: BenchConfig):
    return MazeTask() if bc.task == "maze" else SudokuTask()
