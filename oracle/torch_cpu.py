"""torch (CPU, fp32) restatement of the NCA rollout step -- TEST AND BASELINE INFRASTRUCTURE,
NOT PART OF THE PRODUCT.

The reference computes its rollout with torch: the 3x3 perception as one F.conv2d over the
(B*C, 1, H+2, W+2) padded state with a (heads, 1, 3, 3) weight (src/nca/model.py:175-178), the
MLP as two 1x1 Conv2d layers (src/nca/model.py:277-287), the fire mask from torch.rand on a
generator (src/nca/model.py:567-593), then x + m * dx and the clamp (src/nca/model.py:527-559,
430-438).  This module does the same work with the same torch operators, so that bench.py's CPU
baseline and reference arm time the reference's own way of computing on the host cores (oneDNN
convolutions, torch's thread pool), not a slower numpy loop.  The GPU box does not have the
reference checkout, so the reference cannot be imported there; tests/test_oracle.py checks this
module against the numpy oracle (nca_oracle.py), which is pinned to the reference's golden
vectors.

Only tests/ and bench.py's CPU legs import it.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F


class TorchCpuNca:
    """One model's fp32 parameters as CPU tensors, from oracle.nca_oracle.params_from_arrays."""

    def __init__(self, p: dict, channels: int):
        self.C = channels
        self.taps = torch.from_numpy(np.asarray(p["taps"], np.float32).reshape(-1, 1, 3, 3))
        self.heads = self.taps.shape[0]
        w1 = np.asarray(p["w1"], np.float32)
        w2 = np.asarray(p["w2"], np.float32)
        self.w1 = torch.from_numpy(w1.reshape(w1.shape[0], -1, 1, 1).copy())
        self.b1 = torch.from_numpy(np.asarray(p["b1"], np.float32))
        self.w2 = torch.from_numpy(w2.reshape(w2.shape[0], -1, 1, 1).copy())
        self.b2 = torch.from_numpy(np.asarray(p["b2"], np.float32))
        self.head_w = torch.from_numpy(np.asarray(p["head_w"], np.float32))
        self.head_b = torch.from_numpy(np.asarray(p["head_b"], np.float32))
        self.out_off, self.c_out = int(p["out_off"]), int(p["c_out"])
        self.in_off, self.c_in = int(p["in_off"]), int(np.asarray(p["embed"]).shape[1])
        pad = p.get("pad")
        self.pad = None if pad is None else torch.from_numpy(np.asarray(pad, np.float32))

    def perceive(self, x: torch.Tensor) -> torch.Tensor:
        """(B, C, H, W) -> z (B, heads*C, H, W), head-major, as src/nca/model.py:140-152, 175-178."""
        B, C, H, W = x.shape
        xp = F.pad(x, (1, 1, 1, 1))
        if self.pad is not None:
            v = self.pad[None, :, None]
            xp[:, :, 0, :] = v
            xp[:, :, -1, :] = v
            xp[:, :, :, 0] = v
            xp[:, :, :, -1] = v
        z = F.conv2d(xp.reshape(B * C, 1, H + 2, W + 2), self.taps)
        return z.view(B, C, self.heads, H, W).transpose(1, 2).reshape(B, self.heads * C, H, W)

    def update(self, z: torch.Tensor) -> torch.Tensor:
        return F.conv2d(F.relu(F.conv2d(z, self.w1, self.b1)), self.w2, self.b2)

    def confidence(self, x: torch.Tensor) -> torch.Tensor:
        """Max softmax of the linear head on the readout slice (head 'mlp'), (B, H, W)."""
        out = x[:, self.out_off : self.out_off + self.c_out]
        s = torch.einsum("oc,bchw->bohw", self.head_w, out) + self.head_b[None, :, None, None]
        return torch.softmax(s, dim=1).max(dim=1).values.clamp(0.0, 1.0)

    def step(self, x, given4, clamp, fire) -> torch.Tensor:
        x = x + fire * self.update(self.perceive(x))
        sl = slice(self.in_off, self.in_off + self.c_in)
        x_in = torch.where(given4, clamp, x[:, sl])
        return torch.cat([x[:, : sl.start], x_in, x[:, sl.stop :]], dim=1)


def init_state(inputs: np.ndarray, given: np.ndarray, k: int, channels: int, c_in: int, in_off: int):
    """Zero state with the one-hot clamp of the given cells (src/nca/model.py:384-412, sigma 0):
    x (N*k, C, H, W), given4 (N*k, 1, H, W), clamp (N*k, c_in, H, W)."""
    inp = torch.from_numpy(np.repeat(inputs.astype(np.int64), k, 0))
    gv = torch.from_numpy(np.repeat(given.astype(bool), k, 0))
    B, H, W = inp.shape
    clamp = F.one_hot(inp, c_in).permute(0, 3, 1, 2).float()
    given4 = gv[:, None]
    x = torch.zeros((B, channels, H, W))
    x[:, in_off : in_off + c_in] = torch.where(given4, clamp, x[:, in_off : in_off + c_in])
    return x, given4, clamp


def rollout_steps(model: TorchCpuNca, inputs, given, k: int, n_steps: int, p_fire: float = 0.5,
                  adaptive: tuple[float, float] | None = None, seed: int = 0) -> torch.Tensor:
    """n_steps of the rollout's step loop (src/nca/rollout.py:203-247) on the host cores: one
    torch.rand fire draw per step on a seeded generator, p = p_fire, or with `adaptive`
    (scale, bias) the continuous rule p = scale * (1 - conf) + bias on the cell confidence."""
    x, given4, clamp = init_state(inputs, given, k, model.C, model.c_in, model.in_off)
    gen = torch.Generator().manual_seed(seed)
    B, _, H, W = x.shape
    with torch.no_grad():
        for _ in range(n_steps):
            u = torch.rand((B, 1, H, W), generator=gen)
            if adaptive is None:
                fire = (u < p_fire).float()
            else:
                prob = adaptive[0] * (1.0 - model.confidence(x)[:, None]) + adaptive[1]
                fire = (u < prob).float()
            x = model.step(x, given4, clamp, fire)
    return x
