"""The benchmark configurations' unit figures: FLOP and algorithmic HBM bytes per cell-update
(board x trial x cell x step), the numbers bench.py's roofline divides by, and which ceiling
comes first at the measured peaks."""

import pytest

from ncas_b200.configs import CONFIGS


def test_flop_per_cell_update_is_the_two_gemms():
    # maze: 2 * (128 * 128 + 128 * 32); sudoku: 2 * (256 * 256 + 256 * 64)
    assert CONFIGS["cfg0"].flop_per_cell_update == 40_960
    assert CONFIGS["cfg2"].flop_per_cell_update == 163_840


@pytest.mark.parametrize("name,precision,bytes_", [
    ("cfg2", "bf16", 512),   # hi/lo layout: hi window 128 + lo read 128 + hi, lo writes 256
    ("cfg3", "bf16", 384),   # mirror window 64 + fp32 read 128 + fp32 write 128 + mirror write 64
    ("cfg2", "split", 768),  # fp32 window 256 + fp32 read 256 + fp32 write 256
])
def test_bytes_per_cell_update(name, precision, bytes_):
    assert CONFIGS[name].bytes_per_cell_update(precision) == bytes_


@pytest.mark.parametrize("name,bound", [("cfg2", "tensor"), ("cfg4", "tensor"), ("cfg0", "hbm"),
                                        ("cfg3", "hbm")])
def test_first_ceiling_at_the_measured_peaks(name, bound):
    bc = CONFIGS[name]
    tensor = 1408.2e12 / bc.flop_per_cell_update  # cell-updates/s
    hbm = 6541.8e9 / bc.bytes_per_cell_update("bf16")
    assert ("tensor" if tensor <= hbm else "hbm") == bound


def _bench():
    import importlib.util
    from pathlib import Path

    spec = importlib.util.spec_from_file_location("bench", Path(__file__).resolve().parents[1] / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_bench_roofline_rules():
    # bench.py's roofline: which bytes a launch is charged and which ceiling bounds it
    bench = _bench()
    big = 1 << 33  # a state workspace far larger than L2
    cfg2, cfg3 = CONFIGS["cfg2"], CONFIGS["cfg3"]
    r = bench.roofline(cfg2, "bf16", [500.0], [10**9], [256], False, big)
    assert r["bound"] == "tensor" and r["bytes_per_cell_update"] == 512 and not r["state_in_l2"]
    # streaming 32-channel launches are HBM-bound; resident launches of 20 steps move 10 C / 20 B
    r = bench.roofline(cfg3, "bf16", [100.0], [10**9], [20], False, big)
    assert r["bound"] == "hbm" and r["bytes_per_cell_update"] == 384
    r = bench.roofline(cfg3, "bf16", [100.0], [10**9], [20], True, big)
    assert r["bound"] == "tensor" and r["bytes_per_cell_update"] == 16
    # a one-step launch of the resident configuration streams
    r = bench.roofline(cfg3, "bf16", [100.0, 5.0], [10**9, 5 * 10**7], [20, 1], True, big)
    assert r["bytes_per_cell_update"] == pytest.approx((10**9 * 16 + 5 * 10**7 * 384) / (10**9 + 5 * 10**7))
    # a state that stays in L2 (cfg1's one board) has no HBM ceiling
    r = bench.roofline(CONFIGS["cfg1"], "bf16", [100.0], [10**8], [13000], False, 16 << 20)
    assert r["state_in_l2"] and r["bound"] == "tensor"
