"""nca_b200_run_steps_static: NCA steps for callers that cannot allocate device memory (a
framework whose allocator owns all device memory, a runtime with a device-memory budget fixed at
start-up).  Its scratch is a static device array in the library; these checks
call it through the C ABI and compare it with the allocating path (nca_b200_run_steps on a
caller-allocated state workspace), on two calls in a row with different inputs, so that a call
cannot pass by reusing what the previous call left in the shared array."""

import ctypes as C

import numpy as np
import pytest
import torch

from ncas_b200 import _lib as L
from ncas_b200.configs import build
from ncas_b200.tasks import maze_boards, sudoku_boards

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def fire_desc(masks: torch.Tensor) -> L.NcaFireDesc:
    f = L.NcaFireDesc()
    f.mode = L.FIRE_MASK
    f.masks = masks.data_ptr()
    return f


def allocating_path(eng, batch, x, masks):
    st = eng.new_state(batch.n_inst, batch.hw)
    eng.load_nchw(st, x)
    eng.run(st, batch, masks.shape[0], mode="mask", masks=masks)
    out = eng.store_nchw(st)
    eng.check()
    return out


def static_path(eng, batch, x, masks):
    out = torch.empty_like(x)
    stream = torch.cuda.current_stream(DEV).cuda_stream
    s = L.lib().nca_b200_run_steps_static(
        C.byref(eng.desc), C.byref(batch.desc), eng.prec, x.data_ptr(), out.data_ptr(),
        masks.shape[0], C.byref(fire_desc(masks)), 5000, stream)
    L.check(s, "nca_b200_run_steps_static")
    return out


@pytest.mark.parametrize("task,precision", [("sudoku", "bf16"), ("maze", "split")])
def test_static_scratch_matches_allocating_path_twice(task, precision):
    eng = build(task, seed=0, device=DEV, precision=precision).engine()
    for call in range(2):  # two calls in a row, different inputs each time
        if task == "sudoku":
            boards, K = sudoku_boards(6, seed=10 + call), 4
        else:
            boards, K = maze_boards(3, 19, seed=10 + call), 2
        batch = eng.batch_from_boards(boards.inputs, boards.given, K)
        H, W = boards.shape
        g = torch.Generator(device=DEV).manual_seed(call)
        x = torch.randn((batch.n_inst, eng.channels, H * W), generator=g, device=DEV) * 0.1
        masks = (torch.rand((5, batch.n_inst, H * W), generator=g, device=DEV) < 0.5).to(torch.uint8)
        want = allocating_path(eng, batch, x, masks).cpu().numpy()
        got = static_path(eng, batch, x, masks).cpu().numpy()
        # same kernel, same inputs: identical up to the 2e-2 relative tolerance of the bf16 tests
        # (in practice bit for bit)
        np.testing.assert_allclose(got, want, rtol=0, atol=2e-2 * np.abs(want).max())
        assert np.array_equal(got, want)


def test_static_scratch_rejects_requests_beyond_its_size():
    eng = build("sudoku", seed=0, device=DEV).engine()
    boards = sudoku_boards(300, seed=0)
    batch = eng.batch_from_boards(boards.inputs, boards.given, 2)  # 48,600 cells > 16 MiB of state
    x = torch.zeros((batch.n_inst, 64, 81), device=DEV)
    masks = torch.zeros((1, batch.n_inst, 81), dtype=torch.uint8, device=DEV)
    with pytest.raises(L.NcaError, match="NCA_ERR_SCRATCH"):
        static_path(eng, batch, x, masks)
