"""The k-means restatement (oracle/kmeans.py) against the reference's own
_balanced_spherical_kmeans (src/maple_run/flash_head.py:30-110) run on the
CPU (tests/golden/make_kmeans_golden.py): same initial draw, same labels and
centroids (CPU)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle.kmeans import balanced_kmeans, km_dots, rebalance
from tests.golden.make_kmeans_golden import CASES, unit_rows

GOLD = np.load(Path(__file__).parent / "golden" / "kmeans_golden.npz")


@pytest.mark.parametrize("name", sorted(CASES))
def test_kmeans_restatement_equals_reference(name):
    n, d, c, iters, dseed, _ = CASES[name]
    w = unit_rows(n, d, dseed)
    cent, labels, obj = balanced_kmeans(w, c, GOLD[f"{name}.init"], iters)
    ref_labels = GOLD[f"{name}.labels"]
    assert np.bincount(labels, minlength=c).tolist() == [n // c] * c  # balanced, as the reference's
    np.testing.assert_array_equal(labels, ref_labels)
    # centroids: the same members, summed in another order by the reference
    np.testing.assert_allclose(cent, GOLD[f"{name}.centroids"], rtol=0, atol=2e-6)
    assert 0.0 < obj < 1.0


def test_rebalance_ties_and_order():
    """Eviction keeps the most similar members (lower row on ties) and the
    evicted rows, in ascending order, take the best cluster still open."""
    sims = np.array([[0.9, 0.1], [0.9, 0.2], [0.8, 0.7], [0.5, 0.4]], np.float32)
    labels = np.array([0, 0, 0, 0])
    out = rebalance(sims, labels, 2)
    # rows 0 and 1 tie at 0.9 and are kept; 2 and 3 move to cluster 1
    assert out.tolist() == [0, 0, 1, 1]


def test_dots_are_one_fmaf_chain():
    rs = np.random.default_rng(3)
    a = rs.standard_normal((5, 33)).astype(np.float32)
    b = rs.standard_normal((4, 33)).astype(np.float32)
    got = km_dots(a, b)
    want = np.zeros((5, 4), np.float32)
    for i in range(5):
        for j in range(4):
            acc = np.float32(0)
            for k in range(33):
                acc = np.float32(np.float64(a[i, k]) * np.float64(b[j, k]) + np.float64(acc))
            want[i, j] = acc
    np.testing.assert_array_equal(got, want)
