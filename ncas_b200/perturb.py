"""Host-side draws of test-time perturbations, in the reference's order.

`circular_masks` draws the damage discs of src/nca/perturb.py:42-83 from the rollout's
numpy.random.Generator, with the same draws in the same order (so a seed damages the same cells
as the reference); the state update itself is the library's damage kernel (nca_b200_damage).
`sample_noise` makes the reference's noise draws (src/nca/perturb.py:23-40) on a torch
generator for the "torch" fire stream; the kernel adds the tensor.  With the "philox" stream the
kernel draws the noise itself and nothing here runs.
"""

from __future__ import annotations

import numpy as np
import torch


def sample_noise(B: int, C: int, H: int, W: int, p_t: float, p_s: float, sigma: float,
                 generator: torch.Generator, device) -> torch.Tensor | None:
    """(B, C, H, W) noise of one step, or None when no instance is hit: per instance a draw
    < p_t, per cell a draw < p_s, N(0, sigma^2) values; the generator calls of the reference."""
    if sigma <= 0 or p_t <= 0 or p_s <= 0:
        return None
    active = (torch.rand((B, 1, 1, 1), generator=generator, device=device) < p_t).float()
    if active.sum() == 0:
        return None
    cells = (torch.rand((B, 1, H, W), generator=generator, device=device) < p_s).float()
    noise = torch.randn((B, C, H, W), generator=generator, device=device) * sigma
    return noise * active * cells


def circular_masks(B: int, H: int, W: int, n: int, r_min: float, r_max: float,
                   rng: np.random.Generator, hit: np.ndarray | None = None,
                   geometry: str = "ours") -> np.ndarray:
    """(B, H, W) bool: union of `n` discs per board (boards with hit False are skipped).
    'ours': centres uniform over the grid, radius r ~ U(r_min, r_max) * min(H, W), cells with
    squared distance <= r^2.  'official': cell coordinates spread over [-1, 1], centres uniform in
    [-0.5, 0.5]^2, radius r ~ U(r_min, r_max), squared distance < r^2."""
    masks = np.zeros((B, H, W), dtype=bool)
    if geometry == "official":
        ys = np.linspace(-1.0, 1.0, H)[:, None]
        xs = np.linspace(-1.0, 1.0, W)[None, :]
        for b in range(B):
            if hit is not None and not hit[b]:
                continue
            for _ in range(n):
                cy, cx = rng.uniform(-0.5, 0.5, size=2)
                r = rng.uniform(r_min, r_max)
                masks[b] |= (ys - cy) ** 2 + (xs - cx) ** 2 < r * r
        return masks
    if geometry != "ours":
        raise ValueError(f"unknown damage geometry {geometry!r} (ours | official)")
    yy, xx = np.mgrid[0:H, 0:W]
    scale = min(H, W)
    for b in range(B):
        if hit is not None and not hit[b]:
            continue
        for _ in range(n):
            cy, cx = rng.uniform(0, H), rng.uniform(0, W)
            r = rng.uniform(r_min, r_max) * scale
            masks[b] |= (yy - cy) ** 2 + (xx - cx) ** 2 <= r * r
    return masks
