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
