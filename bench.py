#!/usr/bin/env python
"""Throughput benchmark of the B200 NCA test-time rollout.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg2] [--precision bf16]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N
    python bench.py --impl reference      # the CPU restatement of the reference, host cores

One bench step = one complete rollout of the workload's boards on every rank (weak scaling:
rank r runs its own boards as boards [r * n, (r + 1) * n) of an N-times larger job): state
init, `depth` NCA steps for K trials per board (the persistent tcgen05 step kernel; pruning /
adaptive firing as the workload says), readout and conf@K selection, and for N > 1 the
all-gather of the per-board results.  Inputs are resident in HBM; e2e repeats the step through
the public drop-in API `ncas_b200.rollout.rollout` with boards from host memory and results
copied back.  The metric is cell-updates/s (board x trial x cell x step), whole job.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "cell-updates/sec (board x trial x cell x step)"
UNIT = "cell-updates/s"


def peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def profile_traffic(workload: str) -> float | None:
    """DRAM bytes per cell-update of the step kernel from the committed ncu summary."""
    p = ROOT / "profiles" / f"nca_step_kernel_{workload}.md"
    if not p.exists():
        return None
    m = re.search(r"dram_bytes_per_cell_update\s*=\s*([0-9.eE+-]+)", p.read_text())
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clock/throttle sampling while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict | None:
        rows = [r.split(", ") for r in self.lines if r and r[0].isdigit()]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if len(r) > 5 + i and r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------------------ CPU baseline
def cpu_rollout_rate(bc, boards, n_boards: int, n_steps: int, threads: int):
    """The oracle (numpy restatement of the reference) on a bounded sample of the workload:
    n_boards boards x all K trials x n_steps steps.  Returns (cell-updates/s, sample str)."""
    import oracle.nca_oracle as O
    from ncas_b200.configs import model_config, synthetic_params

    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    cfg = model_config(bc.task)
    p = O.params_from_arrays(synthetic_params(cfg, 0), cfg)
    sub = boards.subset(np.arange(n_boards))
    fire = "adaptive_philox" if bc.adaptive else "philox"
    O.rollout(p, sub.inputs[:1], sub.given[:1], bc.k, 1, channels=cfg.channels, fire=fire, seed=0)  # warm-up
    t0 = time.perf_counter()
    O.rollout(p, sub.inputs, sub.given, bc.k, n_steps, channels=cfg.channels, fire=fire, seed=0)
    dt = time.perf_counter() - t0
    cu = n_boards * bc.k * bc.hw * n_steps
    return cu / dt, f"{n_boards} boards x K={bc.k} x {n_steps} steps ({cu} cell-updates, {dt:.1f} s)"


def cpu_sample_size(bc) -> tuple[int, int]:
    """A sample of roughly 10-20 s of oracle work on a few host cores."""
    per_cu = {"maze": 8.0e-6, "sudoku": 6.0e-6}[bc.task]  # seconds per cell-update on 8 cores, rough
    target = 12.0
    n_boards = max(1, min(bc.n_boards, int(target / (per_cu * bc.k * bc.hw * 8)) or 1))
    steps = max(1, min(bc.depth, int(target / (per_cu * n_boards * bc.k * bc.hw))))
    return n_boards, steps


def run_reference(args) -> None:
    """--impl reference: the reference's algorithm (CPU restatement) on the host cores."""
    from ncas_b200.configs import CONFIGS, boards_for

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    bc = CONFIGS[args.workload]
    boards = boards_for(bc, seed=0, n=min(bc.n_boards, 64))
    threads = os.cpu_count() or 1
    n_boards, steps = cpu_sample_size(bc)
    n_boards = min(n_boards, len(boards))
    for _ in range(args.warmup):
        cpu_rollout_rate(bc, boards, n_boards, max(1, steps // 4), threads)
    rates = []
    sample = ""
    for _ in range(args.steps):
        r, sample = cpu_rollout_rate(bc, boards, n_boards, steps, threads)
        rates.append(r)
    value = float(np.median(rates))
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": n_boards * bc.k * bc.hw * steps / value * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": bc.name, "boards": bc.n_boards, "k": bc.k,
                                        "depth": bc.depth, "hw": bc.hw},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------------- GPU arm
def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from ncas_b200.configs import CONFIGS, boards_for, build, task_for
    from ncas_b200.distributed import gather_results
    from ncas_b200.rollout import RolloutConfig, rollout

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    bc = CONFIGS[args.workload]
    if args.boards or args.depth:
        import dataclasses

        bc = dataclasses.replace(bc, n_boards=args.boards or bc.n_boards, depth=args.depth or bc.depth)
    model = build(bc.task, seed=0, device=dev, precision=args.precision)
    eng = model.engine()
    # Weak scaling: every rank runs the workload's full board count on boards of its own (seed =
    # rank; rank 0's are the one-GPU boards), as global boards [rank * n, (rank + 1) * n) of an
    # N-times larger job, so the Philox streams of all ranks are distinct.
    n_total = bc.n_boards * world
    s = rank * bc.n_boards
    shard = boards_for(bc, seed=rank)
    n, K, HW = len(shard), bc.k, bc.hw
    batch = eng.batch_from_boards(shard.inputs, shard.given, K, inst_offset=s * K)
    st = eng.new_state(n * K, HW)
    updates = torch.zeros(n * K, dtype=torch.int32, device=dev)
    adaptive = (0.9, 0.1) if bc.adaptive else None
    segs = list(range(0, bc.depth, bc.prune_every)) + [bc.depth] if bc.prune_every else [0, bc.depth]
    kern_ms: list[float] = []
    kern_cells: list[int] = []

    def one_step(timed: bool):
        eng.init_state(st, batch)
        for a, b in zip(segs[:-1], segs[1:]):
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev0.record()
            eng.run(st, batch, b - a, mode="adaptive" if adaptive else "philox", p_fire=bc.p_fire,
                    seed=0, step0=a, updates=updates, adaptive=adaptive or (0.9, 0.1))
            ev1.record()
            if timed:
                kern_ms.append((ev0, ev1))
                kern_cells.append(n * K * HW * (b - a))
            if b < bc.depth:
                r = eng.readout(st, batch)
                eng.prune_refill(st, r["pred"], r["board_conf"], n, K, bc.n_cap)
        r = eng.readout(st, batch)
        idx, best, bp = eng.select(r["board_conf"], n, K, pred=r["pred"], hw=HW)
        if world > 1:
            gather_results(best, idx, bp, n_total)
        return best

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        one_step(False)
    eng.check()
    barrier()
    l0 = eng.launches
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        t0.record()
        for _ in range(args.steps):
            one_step(True)
        t1.record()
        barrier()
    eng.check()
    launches = eng.launches - l0
    ms = t0.elapsed_time(t1)
    kdur = [a.elapsed_time(b) for a, b in kern_ms]
    t_max = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    ms = float(t_max.item())
    total_cu = bc.cell_updates * world * args.steps  # all ranks' boards
    value = total_cu / (ms / 1e3)

    # ---- e2e through the public API (host boards in, host results out)
    e2e_value, h2d, d2h = None, 0, 0
    task = task_for(bc)
    rc = RolloutConfig(depth=bc.depth, k=K, fire_rate=bc.p_fire, max_cells=1 << 40,
                       pruning={"every": bc.prune_every, "n_cap": bc.n_cap} if bc.prune_every else None,
                       engine={"fire": "philox", "precision": args.precision,
                               **({"adaptive": {"scale": 0.9, "bias": 0.1}} if bc.adaptive else {})})
    if not args.no_e2e:
        e2e_steps = max(1, min(args.steps, 3))
        rollout(model, task, shard, rc, seed=0, board_offset=s)  # warm-up of the API path
        barrier()
        w0 = time.perf_counter()
        for _ in range(e2e_steps):
            res = rollout(model, task, shard, rc, seed=0, board_offset=s)
        barrier()
        e2e_s = torch.tensor([time.perf_counter() - w0], device=dev)
        if world > 1:
            dist.all_reduce(e2e_s, op=dist.ReduceOp.MAX)
        e2e_value = bc.cell_updates * world * e2e_steps / float(e2e_s.item())
        h2d = int(shard.inputs.nbytes + shard.given.nbytes + shard.targets.nbytes)
        d2h = int(res.pred.size + res.conf.nbytes + res.cell_updates.nbytes)

    if rank == 0:
        pk, pk_kind = peaks()
        flop_per_cu = bc.flop_per_cell_update
        avg_kms = float(np.mean(kdur))
        avg_cells = float(np.mean(kern_cells))
        bytes_per_cu = bc.bytes_per_cell_update(args.precision)
        tb = profile_traffic(bc.name)
        # the roofline of the step kernel is the lower of its two ceilings (cell-updates/s)
        t_peak = pk.get("bf16_tflops_sustained", 1400.0)
        h_peak = pk.get("hbm_gbs", 6650.0)
        t_frac = flop_per_cu * avg_cells / (avg_kms / 1e3) / 1e12 / t_peak
        h_frac = bytes_per_cu * avg_cells / (avg_kms / 1e3) / 1e9 / h_peak
        if t_peak * 1e12 / flop_per_cu <= h_peak * 1e9 / bytes_per_cu:
            roof = {"bound": "tensor", "achieved": t_frac * t_peak, "peak": t_peak,
                    "unit": "TFLOP/s", "frac": t_frac, "peak_kind": f"{pk_kind} bf16 sustained",
                    "other": {"bound": "hbm", "frac": h_frac}}
        else:
            roof = {"bound": "hbm", "achieved": h_frac * h_peak, "peak": h_peak, "unit": "GB/s",
                    "frac": h_frac, "peak_kind": f"{pk_kind} copy bandwidth",
                    "other": {"bound": "tensor", "frac": t_frac}}
        roof.update({"traffic": None if tb is None else tb * avg_cells, "kernel": "nca_step_kernel",
                     "flop_per_cell_update": flop_per_cu, "bytes_per_cell_update": bytes_per_cu})
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16" if args.precision == "bf16" else "bf16x2",
            "data": "synthetic",
            "config": {"workload": bc.name, "boards": n_total, "boards_per_gpu": bc.n_boards, "k": K,
                       "depth": bc.depth,
                       "hw": HW, "task": bc.task, "parallelism": f"{bc.n_boards} boards per GPU on {world} GPU(s)",
                       "l2": f"state {st.buffer.numel() / 1e9:.1f} GB > 126 MB L2 (inputs larger than L2)"},
            "roofline": roof,
            "e2e": None if e2e_value is None else {
                "value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d * world,
                "d2h_bytes_per_step": d2h * world},
            "gpu_launches": launches,
            "clocks": clk.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            nb, stp = cpu_sample_size(bc)
            r_, sample = cpu_rollout_rate(bc, shard, min(nb, len(shard)), stp, os.cpu_count() or 1)
            line["cpu_baseline"] = {"value": r_, "unit": UNIT, "cores": os.cpu_count() or 1,
                                    "kind": "port", "sample": sample}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="cfg2", choices=["cfg0", "cfg1", "cfg2", "cfg3", "cfg4"])
    ap.add_argument("--precision", default="bf16", choices=["bf16", "split"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the public-API (host buffers) pass")
    ap.add_argument("--boards", type=int, default=None, help="smaller case of the workload (profiling)")
    ap.add_argument("--depth", type=int, default=None, help="smaller case of the workload (profiling)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
