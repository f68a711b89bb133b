"""Board-sharded rollout on two GPUs (one process per GPU, NCCL): the gathered per-board results
equal the single-GPU rollout of all boards, bit for bit (the Philox stream is keyed by global
instance, and pruning and selection are rank-local).  Skipped when fewer than two GPUs are
visible."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

N_BOARDS, K, DEPTH = 10, 4, 12


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rc():
    from ncas_b200.rollout import RolloutConfig

    return RolloutConfig(depth=DEPTH, k=K, fire_rate=0.5, pruning={"every": 5, "n_cap": 2},
                         engine={"precision": "split"})


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    from ncas_b200.configs import build
    from ncas_b200.distributed import sharded_rollout
    from ncas_b200.tasks import SudokuTask, sudoku_boards

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        model = build("sudoku", seed=0, device=dev, precision="split")
        out = sharded_rollout(model, SudokuTask(), sudoku_boards(N_BOARDS, seed=3), _rc(), seed=7)
        q.put((rank, out))
    except Exception as ex:  # noqa: BLE001
        q.put((rank, f"error: {type(ex).__name__}: {ex}"))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_sharded_rollout_equals_single_gpu():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    outs = dict(q.get(timeout=300) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for r in range(2):
        assert isinstance(outs[r], dict), outs[r]

    from ncas_b200.configs import build
    from ncas_b200.rollout import rollout, select_best
    from ncas_b200.tasks import SudokuTask, sudoku_boards

    dev = torch.device("cuda", 0)
    model = build("sudoku", seed=0, device=dev, precision="split")
    boards = sudoku_boards(N_BOARDS, seed=3)
    res = rollout(model, SudokuTask(), boards, _rc(), seed=7)
    best = select_best(res.conf, res.alive, K)
    for r in range(2):
        o = outs[r]
        assert np.array_equal(o["best_idx"], best)
        assert np.array_equal(o["best_conf"], res.conf[np.arange(N_BOARDS), best])
        assert np.array_equal(o["answers"], res.pred[np.arange(N_BOARDS), best])
