"""Board sharding and the result all-gather on CPU ranks (gloo, world size 2)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ncas_b200.distributed import gather_results, pack_results, shard_range, unpack_results


def test_shard_ranges_cover_every_board_once():
    for n in (1, 7, 1000):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1


def test_pack_roundtrip():
    conf = torch.tensor([0.25, -1.5, float("inf")])
    idx = torch.tensor([3, 0, 127], dtype=torch.int32)
    ans = torch.randint(0, 10, (3, 81), dtype=torch.uint8)
    c, i, a = unpack_results(pack_results(conf, idx, ans), 81)
    assert torch.equal(c, conf) and torch.equal(i, idx) and torch.equal(a, ans)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, n_boards, q, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        if rank == fail_rank:
            raise RuntimeError("rank failure injected on the host")
        s, e = shard_range(n_boards, world, rank)
        ids = torch.arange(s, e)
        conf = ids.float() / 10
        idx = (ids % 7).to(torch.int32)
        ans = (ids[:, None] + torch.arange(81)[None]).remainder(10).to(torch.uint8)
        c, i, a = gather_results(conf, idx, ans, n_boards)
        q.put((rank, c.numpy(), i.numpy(), a.numpy()))
    except Exception as ex:  # noqa: BLE001
        q.put((rank, "error", type(ex).__name__, str(ex)[:200]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(world, n_boards, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, n_boards, q, fail_rank)) for r in range(world)]
    for p in ps:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda t: t[0])


@pytest.mark.parametrize("n_boards", [9, 1000])
def test_gather_on_two_gloo_ranks(n_boards):
    out = _run(2, n_boards)
    ids = np.arange(n_boards)
    for rank, c, i, a in out:
        np.testing.assert_allclose(c, ids / 10, rtol=1e-6)
        assert np.array_equal(i, ids % 7)
        assert np.array_equal(a, ((ids[:, None] + np.arange(81)[None]) % 10).astype(np.uint8))


def test_failed_rank_is_reported_by_the_others():
    out = _run(2, 10, fail_rank=1)
    assert out[1][1] == "error"
    # rank 0's collective ends with an error (peer gone / timeout) instead of hanging
    assert out[0][1] == "error"


def _sharded_worker(rank, world, port, n_boards, q):
    """sharded_rollout with the per-shard GPU work replaced by a host fake: checks the host
    logic around it (shard ranges, empty shards, the all-gather) on gloo ranks."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import ncas_b200.distributed as D
    from ncas_b200.tasks import sudoku_boards

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    calls = []

    def fake(model, task, shard, rc, seed, board_offset):
        calls.append(len(shard))
        ids = torch.arange(board_offset, board_offset + len(shard))
        ans = torch.from_numpy(shard.inputs.reshape(len(shard), -1).astype(np.uint8))
        return ids.float() / 4, (ids % 3).to(torch.int32), ans

    D._shard_results = fake
    try:
        boards = sudoku_boards(n_boards, seed=1)
        out = D.sharded_rollout(None, None, boards, None, seed=0)
        q.put((rank, calls, out["best_conf"], out["best_idx"], out["answers"]))
    except Exception as ex:  # noqa: BLE001
        q.put((rank, "error", type(ex).__name__, str(ex)[:200], None))
    finally:
        dist.destroy_process_group()


def test_more_ranks_than_boards_gives_empty_shards_that_still_gather():
    world, n_boards = 3, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_sharded_worker, args=(r, world, port, n_boards, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = sorted([q.get(timeout=120) for _ in range(world)], key=lambda t: t[0])
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    from ncas_b200.tasks import sudoku_boards

    boards = sudoku_boards(n_boards, seed=1)
    ids = np.arange(n_boards)
    for rank, calls, conf, idx, ans in out:
        assert calls != "error", (calls, conf, idx)
        # ranks 0 and 1 hold one board each; rank 2's shard is empty and does no shard work
        assert calls == ([] if rank == 2 else [1])
        np.testing.assert_allclose(conf, ids / 4)
        assert np.array_equal(idx, ids % 3)
        assert np.array_equal(ans, boards.inputs.astype(np.uint8))
