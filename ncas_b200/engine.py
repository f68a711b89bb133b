"""Host side of the B200 rollout: weights, batches, states and calls into libnca_b200.

`B200Engine` takes any model object with the reference's layout (nca.model.NCA or
ncas_b200.model.NCA): `cfg`, `perceive.weight`, `update.fc1/fc2`, `head`.  It packs the MLP
weights once into the bf16 shared-memory image the tcgen05 kernels read, and exposes the
operations of the rollout path on device tensors.  All compute is done by the library, called
through its torch operators (torch.ops.nca_b200.*, ncas_b200._ops) on torch's current CUDA
stream; torch provides device memory, the stream and host<->device copies.  Host-side size
queries and the weight packing call the C ABI directly (ctypes).

`B200RolloutBlocks` is the drop-in for nca.engine.inference.UniformRolloutBlocks
(src/nca/engine/inference.py:79-104): same constructor shape and `__call__(x, given4, clamp,
fires, noises)`, selected in the reference's rollout by RolloutConfig.engine.
"""

from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib as L
from ._ops import as_bytes, ops
from .model import FIXED_TAPS, check_supported

# Limit of any single wait inside a kernel (a grid barrier, a pipeline handoff).
DEFAULT_TIMEOUT_MS = int(os.environ.get("NCA_B200_TIMEOUT_MS", "20000"))


def _bf16(a: np.ndarray) -> np.ndarray:
    """Nearest bf16 values (ties to even) of an fp32 array, as fp32."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


@dataclass
class Batch:
    """Device arrays of one batch of instances plus its NcaBatchDesc."""

    desc: L.NcaBatchDesc
    n_inst: int
    height: int
    width: int
    trials: int
    given: torch.Tensor   # (rows, H*W) uint8
    clamp: torch.Tensor   # (rows, H*W, c_in) fp32
    inputs: torch.Tensor  # (rows, H*W) uint8
    inst_row: torch.Tensor | None
    inst_id: torch.Tensor | None = None

    @property
    def hw(self) -> int:
        return self.height * self.width


class State:
    """An NcaState workspace (ping-pong tiled fp32 state, bf16 mirror) owned by torch."""

    def __init__(self, engine: B200Engine, n_inst: int, hw: int):
        lib = L.lib()
        nbytes = C.c_size_t(0)
        L.check(
            lib.nca_b200_state_bytes(n_inst, hw, engine.channels, engine.prec, C.byref(nbytes)),
            "nca_b200_state_bytes",
        )
        self.buffer = torch.empty(int(nbytes.value) + 256, dtype=torch.uint8, device=engine.device)
        base = (self.buffer.data_ptr() + 255) & ~255
        self.st = L.NcaState()
        L.check(
            lib.nca_b200_state_bind(
                C.byref(self.st), base, nbytes.value, n_inst, hw, engine.channels, engine.prec
            ),
            "nca_b200_state_bind",
        )
        self.n_inst, self.hw = n_inst, hw
        self.bytes = as_bytes(self.st)  # the struct as the operators take it


class B200Engine:
    """Weights and library calls of one model on one CUDA device."""

    def __init__(self, model, precision: str = "bf16", device: torch.device | None = None):
        cfg = model.cfg
        check_supported(cfg)
        if precision not in ("bf16", "split"):
            raise ValueError("precision must be 'bf16' or 'split'")
        self.cfg = cfg
        self.precision = precision
        self.prec = L.PREC_BF16 if precision == "bf16" else L.PREC_SPLIT
        w1 = model.update.fc1.weight
        self.device = torch.device(device) if device is not None else w1.device
        if self.device.type != "cuda":
            raise RuntimeError("the b200 backend runs on a CUDA device (no CPU fallback)")
        lib = L.lib()
        self.channels = C_ = cfg.channels
        P = cfg.heads * C_
        Hd = model.update.fc1.weight.shape[0]
        self.hidden = Hd
        w1h = w1.detach().float().reshape(Hd, P).cpu().contiguous().numpy()
        w2h = model.update.fc2.weight.detach().float().reshape(C_, Hd).cpu().contiguous().numpy()
        nbytes = C.c_size_t(0)
        L.check(lib.nca_b200_weights_bytes(C_, P, Hd, C.byref(nbytes)), "nca_b200_weights_bytes")
        img = np.zeros(int(nbytes.value), dtype=np.uint8)
        L.check(
            lib.nca_b200_pack_weights(w1h.ctypes.data, w2h.ctypes.data, C_, P, Hd, img.ctypes.data),
            "nca_b200_pack_weights",
        )
        self.wimg = torch.from_numpy(img).to(self.device)
        self.b1 = model.update.fc1.bias.detach().float().contiguous().to(self.device)
        self.b2 = model.update.fc2.bias.detach().float().contiguous().to(self.device)
        taps = model.perceive.weight.detach().float().reshape(4, 9).cpu().numpy()
        n_out = len(cfg.output_tokens)
        if cfg.head == "l2":  # rows are the output-token embeddings (src/nca/model.py:600-602)
            hw_ = model.out_embed.detach().float().reshape(n_out, cfg.c_out).cpu().numpy()
            hb = np.zeros(n_out, np.float32)
        else:
            hw_ = model.head.weight.detach().float().reshape(n_out, cfg.c_out).cpu().numpy()
            hb = model.head.bias.detach().float().cpu().numpy()
        d = L.NcaModelDesc()
        d.channels, d.perception, d.hidden = C_, P, Hd
        d.c_in, d.in_offset, d.c_out, d.out_offset = cfg.c_in, cfg.in_offset, cfg.c_out, cfg.out_offset
        d.n_out = len(cfg.output_tokens)
        d.fixed_taps = int(np.array_equal(taps.reshape(4, 3, 3), FIXED_TAPS))
        for k in range(4):
            for n in range(9):
                d.taps[k][n] = float(taps[k, n])
        for o in range(d.n_out):
            d.head_b[o] = float(hb[o])
            d.out_tokens[o] = int(cfg.output_tokens[o])
            for c in range(cfg.c_out):
                d.head_w[o][c] = float(hw_[o, c])
        d.head_kind = L.HEAD_L2 if cfg.head == "l2" else L.HEAD_LINEAR
        pad = getattr(model, "pad_vec", None)
        if pad is not None:
            pv = pad.detach().float().cpu().numpy()
            for c in range(C_):
                d.pad[c] = float(pv[c])
        # Split mode with weights that are not bf16 values (trained checkpoints): the image of the
        # residual w - bf16(w) makes the GEMMs fp32-accurate in the weights too.
        self.wimg_lo = None
        if precision == "split":
            r1 = w1h - _bf16(w1h)
            r2 = w2h - _bf16(w2h)
            if np.any(r1) or np.any(r2):
                lo = np.zeros(int(nbytes.value), dtype=np.uint8)
                L.check(lib.nca_b200_pack_weights(np.ascontiguousarray(r1).ctypes.data,
                                                  np.ascontiguousarray(r2).ctypes.data, C_, P, Hd,
                                                  lo.ctypes.data), "nca_b200_pack_weights")
                self.wimg_lo = torch.from_numpy(lo).to(self.device)
                d.weights_lo = self.wimg_lo.data_ptr()
        d.weights = self.wimg.data_ptr()
        d.b1 = self.b1.data_ptr()
        d.b2 = self.b2.data_ptr()
        self.desc = d
        self.desc_bytes = as_bytes(d)
        self.embed = model.embed.detach().float().to(self.device) if hasattr(model, "embed") else None
        self.ctrl = torch.zeros(4, dtype=torch.int32, device=self.device)
        self.timeout_ms = DEFAULT_TIMEOUT_MS
        self.launches = 0  # library kernel launches issued by this engine

    # ------------------------------------------------------------------ batches and states
    def make_batch(
        self,
        given: torch.Tensor,
        clamp: torch.Tensor,
        inputs: torch.Tensor,
        trials: int,
        n_inst: int | None = None,
        inst_offset: int = 0,
        inst_row: torch.Tensor | None = None,
        inst_id: torch.Tensor | None = None,
    ) -> Batch:
        """given (rows, H, W) bool/uint8, clamp (rows, H, W, c_in) fp32, inputs (rows, H, W)
        tokens; instance i uses row inst_row[i] or i // trials, and Philox counters of trial
        inst_offset + inst_id[i] (default inst_offset + i)."""
        rows, H, W = given.shape
        dev = self.device
        g = given.to(dev, torch.uint8).reshape(rows, H * W).contiguous()
        c = clamp.to(dev, torch.float32).reshape(rows, H * W, self.cfg.c_in).contiguous()
        x = inputs.to(dev, torch.uint8).reshape(rows, H * W).contiguous()
        n = rows * trials if n_inst is None else n_inst
        ir = None if inst_row is None else inst_row.to(dev, torch.int32).contiguous()
        iid = None if inst_id is None else inst_id.to(dev, torch.int32).contiguous()
        d = L.NcaBatchDesc()
        d.n_inst, d.height, d.width, d.trials = n, H, W, trials
        d.inst_offset = int(inst_offset)
        d.given, d.clamp, d.inputs = g.data_ptr(), c.data_ptr(), x.data_ptr()
        d.inst_row = _ptr(ir)
        d.inst_id = _ptr(iid)
        b = Batch(d, n, H, W, trials, g, c, x, ir, iid)
        b.bytes = as_bytes(d)
        return b

    def compacted(self, b: Batch, sel: torch.Tensor) -> Batch:
        """The batch of the instances `sel` (increasing) of b: same board rows and Philox trial
        identities, renumbered 0 .. len(sel) - 1 (the compaction of src/nca/rollout.py:262-274)."""
        dev = self.device
        sel = sel.to(dev, torch.int64)
        rows = b.inst_row.long() if b.inst_row is not None else torch.div(
            torch.arange(b.n_inst, device=dev), b.trials, rounding_mode="floor")
        ids = b.inst_id.long() if b.inst_id is not None else torch.arange(b.n_inst, device=dev)
        g = b.given.reshape(-1, b.height, b.width)
        cl = b.clamp.reshape(-1, b.height, b.width, self.cfg.c_in)
        x = b.inputs.reshape(-1, b.height, b.width)
        return self.make_batch(g, cl, x, b.trials, n_inst=int(sel.numel()),
                               inst_offset=b.desc.inst_offset, inst_row=rows[sel], inst_id=ids[sel])

    def batch_from_boards(self, inputs_np: np.ndarray, given_np: np.ndarray, trials: int,
                          inst_offset: int = 0) -> Batch:
        """Boards (N, H, W) tokens / given on the host -> batch of N * trials instances."""
        if self.embed is None:
            raise ValueError("the model has no token embedding")
        inputs = torch.from_numpy(np.ascontiguousarray(inputs_np)).to(self.device)
        given = torch.from_numpy(np.ascontiguousarray(given_np)).to(self.device)
        clamp = self.embed[inputs]  # (N, H, W, c_in) embedding lookup of the input tokens
        return self.make_batch(given, clamp, inputs, trials, inst_offset=inst_offset)

    def new_state(self, n_inst: int, hw: int) -> State:
        return State(self, n_inst, hw)

    def _s(self) -> int:
        return _stream(self.device)

    def init_state(self, st: State, b: Batch) -> None:
        ops().state_init(st.bytes, self.desc_bytes, b.bytes)
        self.launches += 1

    def load_nchw(self, st: State, x: torch.Tensor) -> None:
        x = x.to(self.device, torch.float32).contiguous()
        ops().load_nchw(st.bytes, x)
        self.launches += 1

    def store_nchw(self, st: State, out: torch.Tensor | None = None) -> torch.Tensor:
        H_W = st.hw
        if out is None:
            out = torch.empty((st.n_inst, self.channels, H_W), dtype=torch.float32, device=self.device)
        ops().store_nchw(st.bytes, out)
        self.launches += 1
        return out

    # ------------------------------------------------------------------------- the steps
    def resident_group(self, height: int, width: int) -> int:
        """Whole instances of a height x width board one CTA of the resident kernel keeps in
        shared memory (0: this model shape or board has no resident kernel)."""
        return int(L.lib().nca_b200_resident_group(C.byref(self.desc), int(height), int(width)))

    def run(
        self,
        st: State,
        b: Batch,
        n_steps: int,
        mode: str = "philox",
        p_fire: float = 0.5,
        seed: int = 0,
        step0: int = 0,
        masks: torch.Tensor | None = None,
        uniforms: torch.Tensor | None = None,
        adaptive: tuple[float, float] = (0.9, 0.1),
        updates: torch.Tensor | None = None,
        noise: dict | None = None,
        threshold: tuple[float, float, bool] | None = None,
        resident: bool = False,
    ) -> None:
        """n_steps NCA steps.  mode: 'mask' (masks (n_steps, n_inst, H*W) uint8), 'philox',
        'adaptive' (Philox, p = a * (1 - conf) + b) or 'adaptive_uniform' (uniforms given);
        'threshold' / 'threshold_uniform': the reference's rule with threshold = (p_low, tau,
        given_confident) (p_low for cells with conf > tau, p_fire for the others).
        noise (test-time state noise): {'p_t', 'p_s', 'sigma', 'until'} drawn in the kernel
        from Philox, or {'tensor': (n_inst, C, H*W) fp32} for a single step.
        resident: keep each instance's state in shared memory for all n_steps when whole
        instances fit (bf16 mode below 64 channels without noise or confidence rules; the state
        is kept as bf16 hi + lo parts between the steps), else the streaming kernel."""
        f = L.NcaFireDesc()
        f.mode = {"mask": L.FIRE_MASK, "philox": L.FIRE_PHILOX, "adaptive": L.FIRE_ADAPTIVE_PHILOX,
                  "adaptive_uniform": L.FIRE_ADAPTIVE_UNIFORM, "threshold": L.FIRE_THRESHOLD_PHILOX,
                  "threshold_uniform": L.FIRE_THRESHOLD_UNIFORM}[mode]
        if threshold is not None:
            f.p_low, f.tau, f.given_confident = float(threshold[0]), float(threshold[1]), int(bool(threshold[2]))
        f.p_fire = float(p_fire)
        f.adapt_scale, f.adapt_bias = float(adaptive[0]), float(adaptive[1])
        f.seed = int(seed) & ((1 << 64) - 1)
        f.step0 = int(step0)
        f.resident = int(bool(resident))
        keep = []
        if masks is not None:
            m = masks.to(self.device, torch.uint8).contiguous()
            assert m.numel() == n_steps * b.n_inst * b.hw, "masks must be (n_steps, n_inst, H*W)"
            keep.append(m)
            f.masks = m.data_ptr()
        if uniforms is not None:
            u = uniforms.to(self.device, torch.float32).contiguous()
            assert u.numel() == n_steps * b.n_inst * b.hw
            keep.append(u)
            f.uniforms = u.data_ptr()
        if updates is not None:
            assert updates.dtype == torch.int32 and updates.numel() >= b.n_inst
            f.updates = updates.data_ptr()
        if noise is not None:
            if "tensor" in noise:
                nz = noise["tensor"].to(self.device, torch.float32).contiguous()
                assert n_steps == 1 and nz.numel() == b.n_inst * self.channels * b.hw
                keep.append(nz)
                f.noise_mode, f.noise = L.NOISE_EXTERNAL, nz.data_ptr()
            else:
                f.noise_mode = L.NOISE_PHILOX
                f.noise_p_t, f.noise_p_s = float(noise["p_t"]), float(noise["p_s"])
                f.noise_sigma = float(noise["sigma"])
                f.noise_until = int(noise["until"])
        ops().run_steps(self.desc_bytes, b.bytes, st.bytes, int(n_steps), as_bytes(f), self.ctrl,
                        int(self.timeout_ms))
        self.launches += 1  # the step kernel (the control-word reset is a memset)
        self._keep = keep  # alive until the next call (the kernel reads them asynchronously)

    def check(self) -> None:
        """Synchronise and raise if a kernel reported a failure in the control words."""
        s, detail = ops().ctrl_status(self.ctrl)
        if s != L.NCA_OK:
            raise L.NcaError(s, "kernel", detail)

    # ------------------------------------------------------------------ readout and selection
    def readout(self, st: State, b: Batch, targets: torch.Tensor | None = None,
                want_pred: bool = True, want_cell_conf: bool = False) -> dict[str, torch.Tensor]:
        n, hw = b.n_inst, b.hw
        dev = self.device
        out = {"board_conf": torch.empty(n, dtype=torch.float32, device=dev)}
        if want_pred:
            out["pred"] = torch.empty((n, hw), dtype=torch.uint8, device=dev)
        if want_cell_conf:
            out["cell_conf"] = torch.empty((n, hw), dtype=torch.float32, device=dev)
        tg = None
        if targets is not None:
            tg = targets.to(dev, torch.uint8).reshape(-1, hw).contiguous()
            out["cell_acc"] = torch.empty(n, dtype=torch.float32, device=dev)
            out["exact"] = torch.empty(n, dtype=torch.uint8, device=dev)
        ops().readout(self.desc_bytes, b.bytes, st.bytes, out.get("pred"), out.get("cell_conf"),
                      out["board_conf"], tg, out.get("cell_acc"), out.get("exact"))
        self.launches += 1
        return out

    def select(self, board_conf: torch.Tensor, n_boards: int, trials: int, k_limit: int | None = None,
               alive: torch.Tensor | None = None, pred: torch.Tensor | None = None, hw: int = 0):
        dev = self.device
        idx = torch.empty(n_boards, dtype=torch.int32, device=dev)
        best = torch.empty(n_boards, dtype=torch.float32, device=dev)
        bp = torch.empty((n_boards, hw), dtype=torch.uint8, device=dev) if pred is not None else None
        al = None if alive is None else alive.to(dev, torch.uint8).contiguous()
        ops().select(board_conf.contiguous(), al, n_boards, trials, int(k_limit or trials), idx, best,
                     None if pred is None else pred.contiguous(), hw, bp)
        self.launches += 1
        return idx, best, bp

    def prune_refill(self, st: State, pred: torch.Tensor, board_conf: torch.Tensor, n_boards: int,
                     trials: int, n_cap: int):
        dev = self.device
        src = torch.empty(n_boards * trials, dtype=torch.int32, device=dev)
        kept = torch.empty(n_boards * trials, dtype=torch.uint8, device=dev)
        ops().prune_refill(pred.contiguous(), board_conf.contiguous(), n_boards, trials, pred.shape[-1],
                           int(n_cap), src, kept)
        ops().clone(st.bytes, src)
        self.launches += 2
        return src, kept

    def damage(self, st: State, b: Batch, masks: torch.Tensor) -> None:
        """Damage event: zero state in the cells of masks (rows, H*W) (one mask per board row),
        clamp re-applied (src/nca/rollout.py:206-212)."""
        mk = masks.to(self.device, torch.uint8).contiguous()
        ops().damage(self.desc_bytes, b.bytes, st.bytes, mk)
        self._keep_damage = mk
        self.launches += 1

    def halving(self, pred: torch.Tensor, board_conf: torch.Tensor, rows_per_board: np.ndarray,
                n_cap: int, rng: np.random.Generator) -> torch.Tensor:
        """Niche-Capped Diversity Pruning, halving variant (src/nca/pruning.py:22-65), on the
        alive rows of a compacted batch: board n owns rows_per_board[n] consecutive rows in
        increasing trial order.  Niches and survivors are computed on the device; the host
        draws rng.permutation(n_niches) for every board with more than one alive trial, in
        board order, as the reference does.  Returns keep (rows,) uint8 on the device."""
        dev = self.device
        n = len(rows_per_board)
        rows = int(pred.shape[0])
        starts = np.zeros(n + 1, dtype=np.int32)
        np.cumsum(rows_per_board, out=starts[1:])
        if starts[-1] != rows:
            raise ValueError("rows_per_board does not add up to the batch")
        max_rows = max(1, int(np.max(rows_per_board)) if n else 1)
        row_start = torch.from_numpy(starts).to(dev)
        niche = torch.empty(rows, dtype=torch.int32, device=dev)
        rank = torch.empty(rows, dtype=torch.int32, device=dev)
        n_niches = torch.empty(n, dtype=torch.int32, device=dev)
        hw = int(pred.shape[-1])
        ops().niches(pred.contiguous(), board_conf.contiguous(), row_start, n, max_rows, hw, niche, rank,
                     n_niches)
        nn = n_niches.cpu().numpy()
        order = np.zeros(max(1, int(nn.sum())), dtype=np.int32)
        order_start = np.zeros(n, dtype=np.int32)
        pos = 0
        for b in range(n):
            order_start[b] = pos
            if rows_per_board[b] > 1:
                order[pos : pos + nn[b]] = rng.permutation(int(nn[b]))
            else:
                order[pos : pos + nn[b]] = np.arange(nn[b])
            pos += int(nn[b])
        keep = torch.empty(rows, dtype=torch.uint8, device=dev)
        order_d = torch.from_numpy(order).to(dev)
        order_start_d = torch.from_numpy(order_start).to(dev)
        ops().halving(niche, rank, n_niches, row_start, order_d, order_start_d, n, max_rows, int(n_cap),
                      keep)
        self.launches += 2
        return keep

    def gather(self, st: State, sel: torch.Tensor) -> State:
        """A new state holding the instances `sel` of st (compaction)."""
        sel32 = sel.to(self.device, torch.int32).contiguous()
        dst = self.new_state(int(sel32.numel()), st.hw)
        ops().gather(st.bytes, dst.bytes, sel32)
        self.launches += 1
        return dst

    # ----------------------------------------------------------- reference-shaped NCHW calls
    def _nchw_batch(self, x: torch.Tensor, given4: torch.Tensor, clamp: torch.Tensor) -> Batch:
        B, Cc, H, W = x.shape
        if Cc != self.channels:
            raise ValueError(f"state has {Cc} channels, model {self.channels}")
        given = given4.reshape(B, H, W)
        cl = clamp.to(self.device, torch.float32).permute(0, 2, 3, 1)  # (B, H, W, c_in)
        inputs = torch.zeros((B, H, W), dtype=torch.uint8, device=self.device)
        return self.make_batch(given, cl, inputs, trials=1)

    def step_nchw(self, x, given4, clamp, fire_mask) -> torch.Tensor:
        """NCA.step on reference-layout tensors (src/nca/model.py:503-525)."""
        B, Cc, H, W = x.shape
        b = self._nchw_batch(x, given4, clamp)
        st = self.new_state(B, H * W)
        self.load_nchw(st, x)
        masks = (fire_mask.reshape(1, B, H * W) > 0).to(torch.uint8)
        self.run(st, b, 1, mode="mask", masks=masks)
        return self.store_nchw(st).reshape(B, Cc, H, W)

    def apply_clamp_nchw(self, x, given4, clamp) -> torch.Tensor:
        """NCA.apply_clamp (src/nca/model.py:430-438): a zero-step pass through the state
        layout re-applies nothing, so the clamp is written by loading x and re-initialising the
        given cells' input channels."""
        B, Cc, H, W = x.shape
        b = self._nchw_batch(x, given4, clamp)
        st = self.new_state(B, H * W)
        self.load_nchw(st, x)
        masks = torch.zeros((1, B, H * W), dtype=torch.uint8, device=self.device)
        self.run(st, b, 1, mode="mask", masks=masks)  # no cell fires: x kept, given cells clamped
        return self.store_nchw(st).reshape(B, Cc, H, W)

    def readout_nchw(self, x: torch.Tensor) -> dict[str, torch.Tensor]:
        B, Cc, H, W = x.shape
        given = torch.zeros((B, H, W), dtype=torch.uint8, device=self.device)
        cl = torch.zeros((B, H, W, self.cfg.c_in), dtype=torch.float32, device=self.device)
        b = self.make_batch(given, cl, given, trials=1)
        st = self.new_state(B, H * W)
        self.load_nchw(st, x)
        r = self.readout(st, b, want_pred=True, want_cell_conf=True)
        toks = torch.tensor(self.cfg.output_tokens, device=self.device)
        # pred holds tokens already (no given cells here)
        return {
            "decoded": r["pred"].long().reshape(B, H, W),
            "cell_conf": r["cell_conf"].reshape(B, H, W),
            "board_conf": r["board_conf"],
            "tokens": toks,
        }


class B200RolloutBlocks:
    """Drop-in for nca.engine.inference.UniformRolloutBlocks: runs a block of steps with the
    fire masks the rollout drew, in one persistent launch."""

    def __init__(self, model, config=None, amp: bool = False):
        precision = "bf16"
        if isinstance(config, dict):
            precision = config.get("precision", "bf16")
        elif config is not None:
            precision = getattr(config, "precision", "bf16")
        self.config = config
        self.engine = B200Engine(model, precision=precision)

    def __call__(self, x, given4, clamp, fires, noises):
        if any(n is not None and bool((n != 0).any()) for n in noises):
            raise ValueError("the b200 backend has no step noise")
        e = self.engine
        B, Cc, H, W = x.shape
        b = e._nchw_batch(x, given4, clamp)
        st = e.new_state(B, H * W)
        e.load_nchw(st, x)
        masks = torch.stack([(f.reshape(B, H * W) > 0) for f in fires]).to(torch.uint8)
        e.run(st, b, len(fires), mode="mask", masks=masks)
        return e.store_nchw(st).reshape(B, Cc, H, W)
