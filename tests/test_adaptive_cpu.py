"""Adaptive top-k in the oracle (adaptive_topk.py:44-51, :107-118,
:224-233): the keep rule on hand-checked weight rows and against the keep
counts of the reference's own `_keep_for_mass` (tests/golden/adaptive_keep.npz,
written by make_adaptive_golden.py), the masking of the dropped slots (the
token's first expert, score 0), the renormalisation over the kept mass, and
threshold 1.0 leaving the exact top-k untouched."""
from __future__ import annotations

import os

import numpy as np

import vxmoe_oracle as O


def test_keep_for_mass_matches_reference_counts(golden_dir):
    g = np.load(os.path.join(golden_dir, "adaptive_keep.npz"))
    rows, thresholds, keeps = g["weights"], g["thresholds"], g["keeps"]
    assert keeps.shape == (len(thresholds), len(rows)) and set(np.unique(keeps)) == set(range(1, 11))
    got = np.array([[O.keep_for_mass(r.tolist(), float(t)) for r in rows] for t in thresholds])
    np.testing.assert_array_equal(got, keeps)


def test_keep_for_mass_hand_cases():
    w = [0.5, 0.3, 0.2]
    assert O.keep_for_mass(w, 0.5) == 1          # 0.5 >= 0.5 at the first slot
    assert O.keep_for_mass(w, 0.8) == 2          # 0.5 + 0.3 reaches 0.8
    assert O.keep_for_mass(w, 0.81) == 3
    assert O.keep_for_mass(w, 1.0) == 3
    # the shares are of the row's own sum, not of 1
    assert O.keep_for_mass([2.0, 1.0, 1.0], 0.5) == 1
    assert O.keep_for_mass([1.0, 1.0, 1.0, 1.0], 0.74) == 3
    # a threshold above every running share keeps everything
    assert O.keep_for_mass([0.25] * 4, 1.5) == 4


def test_adaptive_keep_masks_and_min_keep():
    inds = np.array([[7, 3, 9, 1], [4, 5, 6, 8]])
    scores = np.array([[0.6, 0.2, 0.1, 0.1], [0.3, 0.3, 0.2, 0.2]], np.float32)
    ids, kept, keeps = O.adaptive_keep(inds, scores, 0.75)
    assert keeps.tolist() == [2, 3]
    assert ids.tolist() == [[7, 3, 7, 7], [4, 5, 6, 4]]
    assert kept.tolist()[0] == [np.float32(0.6), np.float32(0.2), 0.0, 0.0]
    ids, _, keeps = O.adaptive_keep(inds, scores, 0.5, min_keep=3)
    assert keeps.tolist() == [3, 3]
    ids, kept, keeps = O.adaptive_keep(inds, scores, 1.0)
    assert keeps.tolist() == [4, 4] and np.array_equal(ids, inds) and np.array_equal(kept, scores)
    assert O.keeps_of(O.adaptive_keep(inds, scores, 0.75)[0]).tolist() == [2, 3]


def test_router_adaptive_renormalises_over_kept_mass():
    rng = np.random.default_rng(2)
    logits = O.bf16_round(rng.normal(0, 1, (32, 64)).astype(np.float32))
    exact = O.router(None, None, 8, logits=logits)
    ad = O.router(None, None, 8, logits=logits, threshold=0.6)
    keeps = O.keeps_of(ad.inds)
    assert keeps.min() >= 1 and keeps.mean() < 8
    for t in range(32):
        k = keeps[t]
        np.testing.assert_array_equal(ad.inds[t, :k], exact.inds[t, :k])
        assert np.all(ad.weights[t, k:] == 0)
        # the kept weights renormalise to about 1 (bf16 rounding aside)
        assert abs(float(O.f32(ad.weights[t]).sum()) - 1.0) < 2e-2
    # threshold 1.0 is the exact top-k
    same = O.router(None, None, 8, logits=logits, threshold=1.0)
    np.testing.assert_array_equal(same.inds, exact.inds)
    np.testing.assert_array_equal(same.weights, exact.weights)
