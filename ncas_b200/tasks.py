"""Boards, task metrics and the seeded synthetic board generators of the benchmark configs.

Mirrors the parts of the reference's task layer that the rollout path touches:

* `Boards` -- the (inputs, targets, given) container of src/nca/tasks/base.py:27-86;
* `Task` / `MazeTask` / `SudokuTask` -- eval mask and exact / cell-accuracy metrics
  (src/nca/tasks/base.py:126-143, src/nca/tasks/maze.py:845-867, src/nca/tasks/sudoku.py:987-995);
* maze generators with the same algorithm and the same order of random draws as
  src/nca/tasks/maze.py:317-445 (randomised iterative DFS, endpoint choice, wall removal), so a
  seed gives the same maze as the reference; the second endpoint in row-major order becomes the
  goal token (src/nca/tasks/maze.py:1037-1045);
* sudoku boards as Sudoku-invariant symmetries (src/nca/tasks/sudoku.py:918-943) of a canonical
  solved grid, with a uniformly drawn number of givens.

Host-side numpy only: board generation and scoring are not on the timed path.
"""

from __future__ import annotations

import heapq
from collections import deque
from dataclasses import dataclass, field

import numpy as np

# maze tokens (src/nca/tasks/maze.py:58-59): 0 empty, 1 path, 2 wall, 3 start, 4 goal
EMPTY, PATH, WALL, START, GOAL = 0, 1, 2, 3, 4


@dataclass
class Boards:
    """A batch of boards of one size; all arrays are (N, H, W)."""

    inputs: np.ndarray
    targets: np.ndarray
    given: np.ndarray
    meta: dict = field(default_factory=dict)

    def __post_init__(self) -> None:
        assert self.inputs.shape == self.targets.shape == self.given.shape, "shape mismatch"
        assert self.inputs.ndim == 3, "boards must be (N, H, W)"
        self.inputs = np.asarray(self.inputs).astype(np.int64)
        self.targets = np.asarray(self.targets).astype(np.int64)
        self.given = np.asarray(self.given).astype(bool)

    def __len__(self) -> int:
        return self.inputs.shape[0]

    @property
    def shape(self) -> tuple[int, int]:
        return self.inputs.shape[1], self.inputs.shape[2]

    def subset(self, idx) -> Boards:
        idx = np.asarray(idx)
        meta = {
            k: (v[idx] if isinstance(v, np.ndarray) and v.shape[:1] == (len(self),) else v)
            for k, v in self.meta.items()
        }
        return Boards(self.inputs[idx], self.targets[idx], self.given[idx], meta)

    def repeat(self, k: int) -> Boards:
        meta = {
            key: (np.repeat(v, k, axis=0) if isinstance(v, np.ndarray) and v.shape[:1] == (len(self),) else v)
            for key, v in self.meta.items()
        }
        return Boards(
            np.repeat(self.inputs, k, 0), np.repeat(self.targets, k, 0), np.repeat(self.given, k, 0), meta
        )


class Task:
    """What the rollout needs to know about a benchmark (src/nca/tasks/base.py:89-143)."""

    name = "task"
    vocab_size = 2
    output_tokens: tuple[int, ...] = (0, 1)
    main_metric = "exact"
    fill_given = True

    def eval_mask(self, boards: Boards) -> np.ndarray:
        return ~boards.given

    def cell_accuracy(self, pred: np.ndarray, boards: Boards) -> np.ndarray:
        mask = self.eval_mask(boards)
        correct = (pred == boards.targets) & mask
        return correct.sum(axis=(1, 2)) / np.maximum(mask.sum(axis=(1, 2)), 1)

    def metrics(self, pred: np.ndarray, boards: Boards) -> dict[str, np.ndarray]:
        pred = np.asarray(pred)
        mask = self.eval_mask(boards)
        exact = np.all((pred == boards.targets) | ~mask, axis=(1, 2))
        return {"exact": exact, "cell_acc": self.cell_accuracy(pred, boards)}


class MazeTask(Task):
    name = "maze"
    vocab_size = 5
    output_tokens = (EMPTY, PATH)


class MazeOODTask(Task):
    """Maze-OOD's 4-token vocabulary (src/nca/tasks/maze.py:71, 874-875): both endpoints are
    token 3."""

    name = "maze_ood"
    vocab_size = 4
    output_tokens = (EMPTY, PATH)


class SudokuTask(Task):
    name = "sudoku"
    vocab_size = 10
    output_tokens = tuple(range(1, 10))

    def metrics(self, pred: np.ndarray, boards: Boards) -> dict[str, np.ndarray]:
        out = super().metrics(pred, boards)
        filled = np.where(boards.given, boards.inputs, np.asarray(pred))
        out["valid"] = np.array([sudoku_is_solution(g) for g in filled], dtype=bool)
        return out


# ------------------------------------------------------------------------------------- mazes
def carve_tree(k: int, rng: np.random.Generator) -> np.ndarray:
    """Perfect maze on a k x k lattice by randomised iterative depth-first search.

    Draw order as src/nca/tasks/maze.py:317-351: one integer for the start cell, then one
    uniform per lattice cell up front; the t-th carved edge picks neighbour
    int(u[t] * n_candidates) among the unvisited ones listed up, down, left, right.
    Returns uint8 (2k+1, 2k+1) with lattice cells EMPTY and everything else WALL.
    """
    n = k * k
    grid = np.full((2 * k + 1, 2 * k + 1), WALL, dtype=np.uint8)
    grid[1::2, 1::2] = EMPTY
    if n == 1:
        return grid
    seen = np.zeros(n, dtype=bool)
    cur = int(rng.integers(n))
    seen[cur] = True
    stack = [cur]
    u = rng.random(n).tolist()
    used = 0
    while stack:
        c = stack[-1]
        i, j = divmod(c, k)
        cand = [
            v
            for ok, v in ((i > 0, c - k), (i < k - 1, c + k), (j > 0, c - 1), (j < k - 1, c + 1))
            if ok and not seen[v]
        ]
        if not cand:
            stack.pop()
            continue
        nxt = cand[int(u[used] * len(cand))]
        used += 1
        seen[nxt] = True
        i2, j2 = divmod(nxt, k)
        grid[i + i2 + 1, j + j2 + 1] = EMPTY
        stack.append(nxt)
    return grid


def bfs_dist(passable: np.ndarray, src: tuple[int, int]) -> np.ndarray:
    """4-neighbour BFS distances from src (-1 where unreachable)."""
    H, W = passable.shape
    dist = np.full((H, W), -1, dtype=np.int64)
    dist[src] = 0
    q = deque([src])
    while q:
        i, j = q.popleft()
        d = dist[i, j] + 1
        for a, b in ((i - 1, j), (i + 1, j), (i, j - 1), (i, j + 1)):
            if 0 <= a < H and 0 <= b < W and passable[a, b] and dist[a, b] < 0:
                dist[a, b] = d
                q.append((a, b))
    return dist


def shortest_path(passable: np.ndarray, src, dst) -> list[tuple[int, int]]:
    """One shortest path src -> dst: walk back from dst to a neighbour one step closer, trying
    up, down, left, right.  Unique on perfect mazes."""
    dist = bfs_dist(passable, src)
    assert dist[dst] >= 0, "unreachable"
    H, W = passable.shape
    path = [tuple(dst)]
    i, j = dst
    while dist[i, j] > 0:
        for a, b in ((i - 1, j), (i + 1, j), (i, j - 1), (i, j + 1)):
            if 0 <= a < H and 0 <= b < W and dist[a, b] == dist[i, j] - 1:
                i, j = a, b
                break
        path.append((i, j))
    return path[::-1]


_MOVES = ((-1, 0), (1, 0), (0, -1), (0, 1))  # up, down, left, right


def _walk_back(parent: dict, src, dst) -> list[tuple[int, int]]:
    path = [dst]
    while path[-1] != src:
        path.append(parent[path[-1]])
    return path[::-1]


def bfs_parent_path(passable: np.ndarray, src, dst) -> list[tuple[int, int]]:
    """Shortest path by breadth-first search with parents set on first discovery, neighbours
    tried up, down, left, right, stopping when dst is discovered (the `bfs` targets of
    src/nca/tasks/maze.py:130-160)."""
    H, W = passable.shape
    src, dst = tuple(src), tuple(dst)
    parent = {src: src}
    q = deque([src])
    while q and dst not in parent:
        i, j = q.popleft()
        for di, dj in _MOVES:
            nb = (i + di, j + dj)
            if 0 <= nb[0] < H and 0 <= nb[1] < W and passable[nb] and nb not in parent:
                parent[nb] = (i, j)
                if nb == dst:
                    break
                q.append(nb)
    assert dst in parent, "unreachable"
    return _walk_back(parent, src, dst)


def astar_path(passable: np.ndarray, src, dst) -> list[tuple[int, int]]:
    """Shortest path by A* with the Manhattan heuristic (the `astar` targets of
    src/nca/tasks/maze.py:187-230): the open cell with the smallest f = g + h is expanded
    first, ties broken by the smaller h, then by insertion order; neighbours are tried up, down,
    left, right, and a cell's parent is replaced only by a strictly shorter route."""
    H, W = passable.shape
    src, dst = tuple(src), tuple(dst)
    h = lambda c: abs(c[0] - dst[0]) + abs(c[1] - dst[1])  # noqa: E731
    g = {src: 0}
    parent = {src: src}
    closed = set()
    order = 0
    heap = [(h(src), h(src), order, src)]
    while heap:
        _, _, _, c = heapq.heappop(heap)
        if c in closed:
            continue
        if c == dst:
            return _walk_back(parent, src, dst)
        closed.add(c)
        for di, dj in _MOVES:
            nb = (c[0] + di, c[1] + dj)
            if not (0 <= nb[0] < H and 0 <= nb[1] < W) or not passable[nb] or nb in closed:
                continue
            if nb not in g or g[c] + 1 < g[nb]:
                g[nb] = g[c] + 1
                parent[nb] = c
                order += 1
                heapq.heappush(heap, (g[nb] + h(nb), h(nb), order, nb))
    raise AssertionError("unreachable")


def _with_path(grid: np.ndarray, path, start_tok: int, goal_tok: int) -> np.ndarray:
    t = grid.copy()
    for i, j in path[1:-1]:
        t[i, j] = PATH
    t[path[0]] = start_tok
    t[path[-1]] = goal_tok
    return t


def _goal_second(inputs: np.ndarray, target: np.ndarray, a, b):
    """The endpoint that comes second in row-major order gets the GOAL token."""
    first, second = (a, b) if a < b else (b, a)
    inputs[first], inputs[second] = START, GOAL
    target[first], target[second] = START, GOAL


def perfect_maze(size: int, rng: np.random.Generator, goal: bool = True) -> tuple[np.ndarray, np.ndarray]:
    """A Maze-OOD style maze of odd `size` (draws as src/nca/tasks/maze.py:364-384): a perfect
    maze on the ((size-1)/2)^2 lattice and two distinct random corridor cells as endpoints.
    Returns (inputs, target) uint8 with tokens EMPTY/PATH/WALL/START/GOAL; with goal=False both
    endpoints keep the START (the reference's Maze-OOD ENDPOINT) token, the 4-token vocabulary
    of the maze_ood preset."""
    if size < 5 or size % 2 == 0:
        raise ValueError(f"size must be odd and >= 5, got {size}")
    grid = carve_tree((size - 1) // 2, rng)
    free = np.argwhere(grid == EMPTY)
    ia, ib = rng.choice(len(free), size=2, replace=False)
    a, b = tuple(int(v) for v in free[ia]), tuple(int(v) for v in free[ib])
    path = shortest_path(grid != WALL, a, b)
    target = _with_path(grid, path, START, GOAL)
    inputs = grid.copy()
    if goal:
        _goal_second(inputs, target, a, b)
    else:
        inputs[a], inputs[b] = START, START
        target[a], target[b] = START, START
    return inputs, target


def hard_maze(
    size: int,
    rng: np.random.Generator,
    min_path_len: int = 60,
    extra_openings: float = 0.10,
    max_tries: int = 1000,
    targets: str = "astar",
) -> tuple[np.ndarray, np.ndarray]:
    """A maze with loops (draws as src/nca/tasks/maze.py:387-445): a perfect (size+1)^2 maze,
    a fraction `extra_openings` of the removable interior walls opened, cropped to size x size;
    start = a random corridor cell, goal = a random corridor cell at BFS distance
    >= min_path_len - 1.  The target marks one shortest path, chosen as the reference's Maze-Hard
    task does: `targets` 'astar' (its default) or 'bfs'."""
    path_fn = {"astar": astar_path, "bfs": bfs_parent_path}[targets]
    if size % 2:
        raise ValueError("size must be even")
    k = size // 2
    for _ in range(max_tries):
        grid = carve_tree(k, rng)
        cand = [
            (i, j)
            for i in range(1, 2 * k)
            for j in range(1, 2 * k)
            if (i + j) % 2 == 1 and grid[i, j] == WALL
        ]
        n_open = int(round(extra_openings * len(cand)))
        if n_open > 0:
            for idx in rng.choice(len(cand), size=n_open, replace=False):
                grid[cand[idx]] = EMPTY
        grid = np.ascontiguousarray(grid[:size, :size])
        passable = grid != WALL
        free = np.argwhere(passable)
        for _ in range(5):
            src = tuple(int(v) for v in free[rng.integers(len(free))])
            dist = bfs_dist(passable, src)
            far = np.argwhere(dist >= min_path_len - 1)
            if len(far) == 0:
                continue
            dst = tuple(int(v) for v in far[rng.integers(len(far))])
            target = _with_path(grid, path_fn(passable, src, dst), START, GOAL)
            inputs = grid.copy()
            inputs[src], inputs[dst] = START, GOAL
            return inputs, target
    raise RuntimeError("no maze satisfied min_path_len")


def maze_boards(n: int, size: int, seed: int, hard: bool = False, goal: bool = True, **kw) -> Boards:
    rng = np.random.default_rng(seed)
    ins, tgs = [], []
    for _ in range(n):
        inp, tgt = hard_maze(size, rng, **kw) if hard else perfect_maze(size, rng, goal=goal)
        ins.append(inp)
        tgs.append(tgt)
    inputs = np.stack(ins).astype(np.int64)
    return Boards(inputs, np.stack(tgs).astype(np.int64), inputs != EMPTY, {"seed": seed, "size": size})


# ------------------------------------------------------------------------------------ sudoku
def canonical_solution() -> np.ndarray:
    """A solved 9x9 grid from the band/stack shift pattern: row r is 1..9 rotated left by
    3*(r mod 3) + r // 3."""
    r = np.arange(9)[:, None]
    c = np.arange(9)[None, :]
    return ((3 * (r % 3) + r // 3 + c) % 9 + 1).astype(np.int64)


def sudoku_is_solution(g: np.ndarray) -> bool:
    g = np.asarray(g).reshape(9, 9)
    want = set(range(1, 10))
    rows = all(set(g[i]) == want for i in range(9))
    cols = all(set(g[:, j]) == want for j in range(9))
    boxes = all(set(g[3 * a : 3 * a + 3, 3 * b : 3 * b + 3].ravel()) == want for a in range(3) for b in range(3))
    return rows and cols and boxes


def sudoku_symmetry(rng: np.random.Generator):
    """(row_perm, col_perm, transpose, digit_perm), draws as src/nca/tasks/sudoku.py:918-927:
    rows permuted within bands and bands permuted, the same for columns, a coin for the
    transpose and a permutation of the digits."""

    def within_bands() -> np.ndarray:
        bands = rng.permutation(3)
        return np.concatenate([3 * b + rng.permutation(3) for b in bands])

    digits = np.concatenate([[0], rng.permutation(9) + 1])
    return within_bands(), within_bands(), bool(rng.integers(2)), digits


def apply_symmetry(grid, row_perm, col_perm, transpose, digit_perm=None) -> np.ndarray:
    g = np.asarray(grid)
    if transpose:
        g = g.T
    g = g[row_perm][:, col_perm]
    if digit_perm is not None:
        g = np.asarray(digit_perm)[g]
    return g


def sudoku_boards(n: int, seed: int, clues: tuple[int, int] = (17, 35), canonical=None) -> Boards:
    """n valid boards: a random symmetry of `canonical`, then a uniform number of givens in
    [clues[0], clues[1]] at uniformly random cells."""
    rng = np.random.default_rng(seed)
    base = canonical_solution() if canonical is None else np.asarray(canonical, dtype=np.int64)
    sols, givens = [], []
    for _ in range(n):
        sol = apply_symmetry(base, *sudoku_symmetry(rng))
        kk = int(rng.integers(clues[0], clues[1] + 1))
        mask = np.zeros(81, dtype=bool)
        mask[rng.choice(81, kk, replace=False)] = True
        sols.append(sol)
        givens.append(mask.reshape(9, 9))
    targets = np.stack(sols)
    given = np.stack(givens)
    return Boards(np.where(given, targets, 0), targets, given, {"seed": seed})
