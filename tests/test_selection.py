"""conf@K, pass@K and niche-capped pruning of the oracle against the reference."""

import numpy as np

import oracle.nca_oracle as O


def test_conf_and_pass_at_k_match_reference(golden):
    ks = [1, 2, 4, 8]
    ck = O.conf_at_k(golden["sel_metric"], golden["sel_conf"], golden["sel_alive"], ks)
    pk = O.pass_at_k(golden["sel_metric"], golden["sel_alive"], ks)
    np.testing.assert_allclose([ck[k] for k in ks], golden["sel_confk"])
    np.testing.assert_allclose([pk[k] for k in ks], golden["sel_passk"])


def test_conf_at_k_known_answer():
    """tests/test_rollout.py:63-71 of the reference."""
    metric = np.array([[True, False, False], [False, False, True]])
    conf = np.array([[0.1, 0.9, 0.5], [0.2, 0.3, 0.9]])
    alive = np.ones((2, 3), dtype=bool)
    assert O.conf_at_k(metric, conf, alive, [1, 2, 3]) == {1: 0.5, 2: 0.0, 3: 0.5}
    assert O.pass_at_k(metric, alive, [1, 3]) == {1: 0.5, 3: 1.0}


def test_halving_pruning_matches_reference(golden):
    rng = np.random.default_rng(42)
    new = O.niche_capped_pruning(golden["prune_dec"], golden["prune_conf"], golden["prune_alive"], 2,
                                 lambda n: rng.permutation(n))
    assert np.array_equal(new, golden["prune_new"])


def test_halving_pruning_known_answer():
    """tests/test_model.py:165-177 of the reference: 2 niches of 4 -> 2 survivors each."""
    dec = np.zeros((1, 8, 2, 2), dtype=np.int64)
    dec[0, 4:] = 1
    conf = np.array([[0.9, 0.8, 0.7, 0.6, 0.5, 0.4, 0.3, 0.2]])
    rng = np.random.default_rng(0)
    new = O.niche_capped_pruning(dec, conf, np.ones((1, 8), bool), 3, lambda n: rng.permutation(n))
    assert new.sum() == 4 and new[0, :4].sum() == 2 and new[0, 4:].sum() == 2
    assert new[0, 0] and new[0, 4]


def test_refill_keeps_top_of_each_niche_and_clones_best():
    dec = np.zeros((1, 8, 4), dtype=np.int64)
    dec[0, 4:] = 1                     # two niches of 4
    dec[0, 7] = 2                      # ... and a singleton
    conf = np.array([[0.9, 0.8, 0.7, 0.6, 0.5, 0.95, 0.3, 0.2]], dtype=np.float32)
    src, kept = O.niche_cap_refill(dec, conf, 2)
    assert kept[0].tolist() == [True, True, False, False, True, True, False, True]
    # kept ranked by confidence: 5 (0.95), 0 (0.9), 1 (0.8), 4 (0.5), 7 (0.2)
    assert src[0].tolist() == [0, 1, 5, 0, 4, 5, 1, 7]


def test_refill_ties_go_to_the_lower_trial():
    dec = np.zeros((1, 4, 3), dtype=np.int64)
    conf = np.full((1, 4), 0.5, dtype=np.float32)
    src, kept = O.niche_cap_refill(dec, conf, 2)
    assert kept[0].tolist() == [True, True, False, False]
    assert src[0].tolist() == [0, 1, 0, 1]
