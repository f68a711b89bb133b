"""Host-side perturbation draws and the threshold firing rule against the reference's own outputs
(tests/golden/golden.npz, made by tests/golden/make_golden.py from the reference)."""

import numpy as np
import torch

import oracle.nca_oracle as O
from ncas_b200.configs import model_config, synthetic_params
from ncas_b200.perturb import circular_masks, sample_noise


def test_damage_discs_match_reference(golden):
    ours = circular_masks(4, 15, 13, 2, 0.1, 0.4, np.random.default_rng(21))
    assert np.array_equal(ours, golden["dmg_ours"])
    off = circular_masks(3, 9, 9, 1, 0.2, 0.5, np.random.default_rng(22), geometry="official")
    assert np.array_equal(off, golden["dmg_official"])


def test_noise_draws_match_reference(golden):
    nz = sample_noise(6, 8, 5, 5, 0.6, 0.5, 0.05, torch.Generator().manual_seed(7), "cpu")
    assert nz is not None and np.array_equal(nz.numpy(), golden["noise_draw"])
    assert sample_noise(6, 8, 5, 5, 0.0, 0.5, 0.05, torch.Generator(), "cpu") is None


def test_threshold_rule_matches_reference(golden):
    """The oracle's threshold rule (the kernel's, src/nca/model.py:566-593) applied to the
    reference's own uniforms gives the reference's masks, with and without given_confident."""
    cfg = model_config("sudoku")
    p = O.params_from_arrays(synthetic_params(cfg, 0), cfg)
    x = golden["thr_x"]
    u = golden["thr_u"][:, 0]
    conf = O.confidence(x, p)
    given = golden["thr_given"][:, 0]
    for mask, gc in ((golden["thr_mask"], False), (golden["thr_mask_given"], True)):
        confident = conf > np.float32(0.12)
        if gc:
            confident = confident | given
        got = u < np.where(confident, np.float32(0.1), np.float32(0.5))
        assert np.array_equal(got, mask[:, 0] > 0)
