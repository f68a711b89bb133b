#!/usr/bin/env python
"""Throughput benchmark of the B200 NCA test-time rollout.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg2] [--precision bf16]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N
    python bench.py --impl reference      # the reference's step loop in torch fp32, host cores

One bench step = one complete rollout of the workload's boards, split evenly over the ranks with
all K trials of a board on one rank (strong scaling; --scaling weak gives every rank the full
board count instead): state init, `depth` NCA steps for K trials per board (the persistent
tcgen05 step kernel; pruning / adaptive firing as the workload says), readout and conf@K
selection, and for N > 1 the all-gather of the per-board results.  Inputs are resident in HBM;
e2e repeats the step through the public drop-in API `ncas_b200.rollout.rollout` with boards from
host memory and results copied back.  The metric is cell-updates/s (board x trial x cell x
step), whole job.  The line also carries `split`: the same workload in the parity precision.
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
        if self.gpu is None:
            return self
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
            # a timed region shorter than nvidia-smi's start-up and 200 ms period (cfg0)
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "note": "timed region shorter than the 200 ms sampling period"}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if len(r) > 5 + i and r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------------------ CPU baseline
def _host_threads() -> int:
    """All host cores, whatever torchrun exported: torch's pool and the BLAS pools are set
    explicitly (torchrun sets OMP_NUM_THREADS=1 for every rank)."""
    n = os.cpu_count() or 1
    import torch

    torch.set_num_threads(n)
    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(limits=n)
    except ImportError:
        pass
    return n


def cpu_rollout_rate(bc, boards, budget_s: float = 12.0):
    """The reference's step loop computed with torch on the host cores (oracle/torch_cpu.py:
    F.conv2d perception, 1x1-conv MLP, torch.rand fire draws, fp32), on a bounded sample of the
    workload: a few boards x all K trials x enough steps for about `budget_s` seconds.
    Returns (cell-updates/s, sample description, threads)."""
    import oracle.nca_oracle as O
    import oracle.torch_cpu as TC
    from ncas_b200.configs import model_config, synthetic_params

    threads = _host_threads()
    cfg = model_config(bc.task)
    m = TC.TorchCpuNca(O.params_from_arrays(synthetic_params(cfg, 0), cfg), cfg.channels)
    adaptive = (0.9, 0.1) if bc.adaptive else None
    # a few boards: about 50k-100k cells per step, like the reference's own per-pass batches
    n_boards = max(1, min(len(boards), 100_000 // (bc.k * bc.hw)))
    sub = boards.subset(np.arange(n_boards))
    TC.rollout_steps(m, sub.inputs, sub.given, bc.k, 1, bc.p_fire, adaptive)  # warm-up
    t0 = time.perf_counter()
    TC.rollout_steps(m, sub.inputs, sub.given, bc.k, 2, bc.p_fire, adaptive)
    per_step = (time.perf_counter() - t0) / 2
    steps = max(2, min(bc.depth, int(budget_s / max(per_step, 1e-6))))
    t0 = time.perf_counter()
    TC.rollout_steps(m, sub.inputs, sub.given, bc.k, steps, bc.p_fire, adaptive)
    dt = time.perf_counter() - t0
    cu = n_boards * bc.k * bc.hw * steps
    sample = (f"{n_boards} boards x K={bc.k} x {steps} steps of {bc.name} ({cu} cell-updates, "
              f"{dt:.1f} s, torch fp32 on {threads} threads)")
    return cu / dt, sample, threads


def run_reference(args) -> None:
    """--impl reference: the reference's step loop as the reference computes it (torch fp32
    operators on the host cores), rank 0 only."""
    from ncas_b200.configs import CONFIGS, boards_for

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    bc = CONFIGS[args.workload]
    boards = boards_for(bc, seed=0, n=min(bc.n_boards, 64))
    for _ in range(args.warmup):
        cpu_rollout_rate(bc, boards, budget_s=1.0)
    rates = []
    sample, threads = "", 1
    for _ in range(args.steps):
        r, sample, threads = cpu_rollout_rate(bc, boards, budget_s=4.0)
        rates.append(r)
    value = float(np.median(rates))
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": bc.cell_updates / value * 1e3,
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": bc.name, "boards": bc.n_boards, "k": bc.k,
                                        "depth": bc.depth, "hw": bc.hw},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------------- GPU arm
L2_BYTES = 126 * 1024 * 1024  # B200 L2


def roofline(bc, precision: str, kdur_ms: list[float], cells: list[int], steps: list[int],
             resident: bool, state_bytes: int) -> dict:
    """The step kernel's roofline from its CUDA-event launch times: the lower of the tensor
    ceiling (GEMM FLOPs) and the HBM ceiling (algorithmic bytes) per cell-update.  cells: the
    cell-updates of each launch, steps: its steps; resident: the launches with more than one
    step ran the shared-memory-resident kernel, which reads the fp32 state once (4C bytes per
    cell) and writes it and its bf16 copy once (6C) per launch.  A state workspace of at most
    half the L2 stays in L2 from step to step (cfg1's one board), so no HBM ceiling applies to
    it: the bound is then the tensor pipe."""
    pk, pk_kind = peaks()
    flop_per_cu = bc.flop_per_cell_update
    # split mode runs every GEMM on the hi and the lo part of its activations: twice the MMAs
    executed = flop_per_cu * (2 if precision == "split" else 1)
    avg_kms = float(np.mean(kdur_ms))
    avg_cells = float(np.mean(cells))
    stream_b = bc.bytes_per_cell_update(precision)
    per_launch = [c * (10 * bc.channels / n if resident and n > 1 else stream_b) for c, n in zip(cells, steps)]
    bytes_per_cu = float(sum(per_launch)) / float(sum(cells))
    tb = profile_traffic(bc.name) if precision == "bf16" else None
    t_peak = pk.get("bf16_tflops_sustained", 1400.0)
    t_burst = pk.get("bf16_tflops", 1590.0)
    h_peak = pk.get("hbm_gbs", 6650.0)
    t_ach = flop_per_cu * avg_cells / (avg_kms / 1e3) / 1e12
    t_frac = t_ach / t_peak
    h_frac = bytes_per_cu * avg_cells / (avg_kms / 1e3) / 1e9 / h_peak
    l2_resident = state_bytes <= L2_BYTES // 2
    if l2_resident or t_peak * 1e12 / executed <= h_peak * 1e9 / bytes_per_cu:
        roof = {"bound": "tensor", "achieved": t_ach, "peak": t_peak, "unit": "TFLOP/s",
                "frac": t_frac, "peak_kind": f"{pk_kind} bf16 sustained",
                "frac_of_burst": t_ach / t_burst, "other": {"bound": "hbm", "frac": h_frac}}
    else:
        roof = {"bound": "hbm", "achieved": h_frac * h_peak, "peak": h_peak, "unit": "GB/s",
                "frac": h_frac, "peak_kind": f"{pk_kind} copy bandwidth",
                "other": {"bound": "tensor", "frac": t_frac}}
    if precision == "split":
        roof["executed_tflops"] = executed * avg_cells / (avg_kms / 1e3) / 1e12
    roof.update({"traffic": None if tb is None else tb * avg_cells, "kernel": "nca_step_kernel",
                 "flop_per_cell_update": flop_per_cu, "bytes_per_cell_update": bytes_per_cu,
                 "kernel_ms": avg_kms, "resident": resident, "state_in_l2": l2_resident})
    return roof


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from ncas_b200.configs import CONFIGS, boards_for, build, task_for
    from ncas_b200.distributed import gather_results, shard_range
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
    # Strong scaling (default): the workload's boards are split evenly over the ranks, all K
    # trials of a board on one rank, as one job.  Weak scaling: every rank runs the workload's
    # board count on boards of its own (global boards [rank * n, (rank + 1) * n) of an N-times
    # larger job).  A workload with fewer boards than ranks (cfg1) runs replicas (weak).
    scaling = args.scaling if bc.n_boards >= world else "weak"
    if scaling == "strong":
        n_total = bc.n_boards
        s, e = shard_range(n_total, world, rank)
        shard = boards_for(bc, seed=0).subset(np.arange(s, e))
    else:
        n_total = bc.n_boards * world
        s = rank * bc.n_boards
        shard = boards_for(bc, seed=rank)
    n, K, HW = len(shard), bc.k, bc.hw
    total_cu = n_total * K * HW * bc.depth  # all ranks' cell-updates of one bench step
    adaptive = (0.9, 0.1) if bc.adaptive else None
    segs = list(range(0, bc.depth, bc.prune_every)) + [bc.depth] if bc.prune_every else [0, bc.depth]

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(v: float) -> float:
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def measure(precision: str, steps: int, warmup: int, clocks: bool):
        """`warmup` then `steps` timed bench steps of the workload in `precision`: returns
        (ms of the timed region (max over ranks), step-kernel event pairs, their cell-updates,
        library launches, clock summary, state bytes)."""
        model = build(bc.task, seed=0, device=dev, precision=precision)
        eng = model.engine()
        batch = eng.batch_from_boards(shard.inputs, shard.given, K, inst_offset=s * K)
        st = eng.new_state(n * K, HW)
        updates = torch.zeros(n * K, dtype=torch.int32, device=dev)
        kern, kern_cells, kern_steps = [], [], []

        def one_step(timed: bool):
            eng.init_state(st, batch)
            for a, b in zip(segs[:-1], segs[1:]):
                ev0 = torch.cuda.Event(enable_timing=True)
                ev1 = torch.cuda.Event(enable_timing=True)
                ev0.record()
                eng.run(st, batch, b - a, mode="adaptive" if adaptive else "philox", p_fire=bc.p_fire,
                        seed=0, step0=a, updates=updates, adaptive=adaptive or (0.9, 0.1),
                        resident=not args.no_resident)
                ev1.record()
                if timed:
                    kern.append((ev0, ev1))
                    kern_cells.append(n * K * HW * (b - a))
                    kern_steps.append(b - a)
                if b < bc.depth:
                    r = eng.readout(st, batch)
                    eng.prune_refill(st, r["pred"], r["board_conf"], n, K, bc.n_cap)
            r = eng.readout(st, batch)
            idx, best, bp = eng.select(r["board_conf"], n, K, pred=r["pred"], hw=HW)
            if world > 1:
                gather_results(best, idx, bp, n_total)

        for _ in range(warmup):
            one_step(False)
        eng.check()
        barrier()
        l0 = eng.launches
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        with ClockSampler(local if clocks else None) as clk:
            barrier()
            t0.record()
            for _ in range(steps):
                one_step(True)
            t1.record()
            barrier()
        eng.check()
        ms = max_over_ranks(t0.elapsed_time(t1))
        kdur = [a.elapsed_time(b) for a, b in kern]
        res = (precision == "bf16" and not adaptive and not args.no_resident
               and eng.resident_group(shard.inputs.shape[1], shard.inputs.shape[2]) >= 1)
        return ms, kdur, (kern_cells, kern_steps, res), eng.launches - l0, clk.summary(), st.buffer.numel(), model

    ms, kdur, kcells, launches, clocks, state_bytes, model = measure(args.precision, args.steps,
                                                                     args.warmup, True)
    value = total_cu * args.steps / (ms / 1e3)

    # ---- e2e through the public API (host boards in, host results out)
    e2e_value, h2d, d2h = None, 0, 0
    task = task_for(bc)
    rc = RolloutConfig(depth=bc.depth, k=K, fire_rate=bc.p_fire, max_cells=1 << 40,
                       pruning={"every": bc.prune_every, "n_cap": bc.n_cap} if bc.prune_every else None,
                       engine={"fire": "philox", "precision": args.precision, "resident": not args.no_resident,
                               **({"adaptive": {"scale": 0.9, "bias": 0.1}} if bc.adaptive else {})})
    if not args.no_e2e:
        e2e_steps = max(1, min(args.steps, 3))
        rollout(model, task, shard, rc, seed=0, board_offset=s)  # warm-up of the API path
        barrier()
        w0 = time.perf_counter()
        for _ in range(e2e_steps):
            res = rollout(model, task, shard, rc, seed=0, board_offset=s)
        barrier()
        e2e_s = max_over_ranks(time.perf_counter() - w0)
        e2e_value = total_cu * e2e_steps / e2e_s
        io = torch.tensor([shard.inputs.nbytes + shard.given.nbytes + shard.targets.nbytes,
                           res.pred.size + res.conf.nbytes + res.cell_updates.nbytes],
                          dtype=torch.int64, device=dev)
        if world > 1:
            dist.all_reduce(io)
        h2d, d2h = int(io[0]), int(io[1])

    # ---- the parity mode (fp32 stencil, GEMMs on bf16 hi + lo parts) on the same workload
    split = None
    if args.precision == "bf16" and not args.no_split:
        sms, skdur, skcells, _, _, sstate, _ = measure("split", max(1, min(args.steps, 3)), 1, False)
        split = {"value": total_cu * max(1, min(args.steps, 3)) / (sms / 1e3),
                 "ms_per_step": sms / max(1, min(args.steps, 3)),
                 "roofline": roofline(bc, "split", skdur, *skcells, sstate)}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None, "dtype": "bf16" if args.precision == "bf16" else "bf16x2",
            "data": "synthetic",
            "config": {"workload": bc.name, "boards": n_total, "boards_per_gpu": n, "k": K,
                       "depth": bc.depth, "hw": HW, "task": bc.task, "precision": args.precision,
                       "resident": not args.no_resident,
                       "parallelism": f"{n_total} boards over {world} GPU(s), all K trials of a board on one GPU",
                       "l2": f"state {state_bytes / 1e9:.2f} GB per GPU vs 126 MB L2"},
            "roofline": roofline(bc, args.precision, kdur, *kcells, state_bytes),
            "e2e": None if e2e_value is None else {
                "value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches,
            "clocks": clocks,
        }
        if split is not None:
            line["split"] = split
        if world == 1 and not args.no_cpu_baseline:
            r_, sample, threads = cpu_rollout_rate(bc, shard)
            line["cpu_baseline"] = {"value": r_, "unit": UNIT, "cores": threads, "kind": "port",
                                    "sample": sample}
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
    ap.add_argument("--no-split", action="store_true", help="skip the split-precision measurement")
    ap.add_argument("--no-resident", action="store_true",
                    help="stream every step through HBM (no shared-memory-resident kernel)")
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"],
                    help="strong: the workload's boards split over the GPUs; weak: every GPU runs them")
    ap.add_argument("--boards", type=int, default=None, help="smaller case of the workload (profiling)")
    ap.add_argument("--depth", type=int, default=None, help="smaller case of the workload (profiling)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
