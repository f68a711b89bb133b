"""Board-sharded rollouts over several GPUs (one process per GPU, torch.distributed).

Boards are independent, so they are split into contiguous shards, all K trials of a board on
the same rank: pruning, refill and conf@K selection stay local.  The only exchange is one
all-gather of the per-board results (best confidence, best trial, decoded answer), packed into a
single byte tensor per rank.  The reference has no distributed code; this replaces running its
rollout (src/nca/rollout.py:86-305) over the whole board set in one process.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist


def shard_range(n_boards: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous shard of rank `rank`: sizes differ by at most one, larger shards first."""
    base, extra = divmod(n_boards, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def pack_results(best_conf: torch.Tensor, best_idx: torch.Tensor, answers: torch.Tensor) -> torch.Tensor:
    """(n,) fp32, (n,) int32, (n, hw) uint8 -> (n, 8 + hw) uint8 rows."""
    n = best_conf.shape[0]
    head = torch.stack([best_conf.float().contiguous().view(torch.int32), best_idx.to(torch.int32)], dim=1)
    return torch.cat([head.contiguous().view(torch.uint8).reshape(n, 8),
                      answers.to(torch.uint8).reshape(n, answers.shape[-1])], 1)


def unpack_results(rows: torch.Tensor, hw: int):
    head = rows[:, :8].contiguous().view(torch.int32).reshape(-1, 2)
    return head[:, 0].contiguous().view(torch.float32), head[:, 1].clone(), rows[:, 8 : 8 + hw].clone()


def gather_results(best_conf, best_idx, answers, n_boards: int, group=None):
    """All-gather the per-board results of every rank's shard; returns the full
    (best_conf (N,), best_idx (N,), answers (N, hw)) on every rank, in board order."""
    world = dist.get_world_size(group)
    hw = answers.shape[1]
    rows = pack_results(best_conf, best_idx, answers)
    max_n = shard_range(n_boards, world, 0)[1]
    pad = torch.zeros((max_n, rows.shape[1]), dtype=torch.uint8, device=rows.device)
    pad[: rows.shape[0]] = rows
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad, group=group)
    parts = []
    for r in range(world):
        s, e = shard_range(n_boards, world, r)
        parts.append(bufs[r][: e - s])
    return unpack_results(torch.cat(parts, 0), hw)


def _shard_results(model, task, shard, rc, seed: int, board_offset: int):
    """Rollout of one rank's (non-empty) shard and its conf@K selection on the rank's GPU:
    (best_conf (n,), best_idx (n,), answers (n, hw)) device tensors."""
    from .rollout import rollout

    res = rollout(model, task, shard, rc, seed=seed, board_offset=board_offset)
    eng = model._engine
    n, K, H, W = res.pred.shape
    dev = eng.device
    conf = torch.from_numpy(res.conf).to(dev)
    alive = torch.from_numpy(res.alive.astype(np.uint8)).to(dev)
    pred = torch.from_numpy(res.pred.reshape(n * K, H * W).astype(np.uint8)).to(dev)
    idx, best, ans = eng.select(conf.reshape(-1), n, K, alive=alive.reshape(-1), pred=pred, hw=H * W)
    return best, idx, ans


def _result_device(group) -> torch.device:
    """Where a rank keeps the tensors it all-gathers: host memory for gloo, else its GPU."""
    if dist.is_initialized() and dist.get_backend(group) == "gloo":
        return torch.device("cpu")
    return torch.device("cuda", torch.cuda.current_device())


def sharded_rollout(model, task, boards, rc, seed: int = 0, group=None):
    """Every rank rolls out its shard of `boards` on its current CUDA device, selects the
    conf@K trial per board with the library's selection kernel, and all ranks receive the
    results of every board: dict(best_conf, best_idx, answers) as numpy arrays.  A rank whose
    shard is empty (more ranks than boards) launches nothing and joins the all-gather with
    zero rows."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    s, e = shard_range(len(boards), world, rank)
    H, W = boards.shape
    if e > s:
        best, idx, ans = _shard_results(model, task, boards.subset(np.arange(s, e)), rc, seed, s)
    else:
        dev = _result_device(group)
        best = torch.zeros(0, dtype=torch.float32, device=dev)
        idx = torch.zeros(0, dtype=torch.int32, device=dev)
        ans = torch.zeros((0, H * W), dtype=torch.uint8, device=dev)
    if world > 1:
        best, idx, ans = gather_results(best, idx, ans, len(boards), group)
    return {
        "best_conf": best.cpu().numpy(),
        "best_idx": idx.cpu().numpy(),
        "answers": ans.cpu().numpy().reshape(-1, H, W),
    }
