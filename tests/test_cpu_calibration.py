"""The calibration oracle on the CPU: its band is numpy's quantile (the
reference's own call) and its exact k-means never has a larger SSE than
sklearn's KMeans (the reference's clusterer, n_init = 3) on the
distributions a KV channel shows, ties and heavy tails included."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import calibrate as oc


def _samples(kind, n, rng):
    if kind == "normal":
        return rng.standard_normal(n)
    if kind == "heavy":
        return rng.standard_t(3, n)
    if kind == "bimodal":
        return np.concatenate([rng.normal(-3, 0.5, n // 2), rng.normal(2, 1.0, n - n // 2)])
    return np.round(rng.standard_normal(n) * 4) / 4          # few distinct values, many ties


@pytest.mark.parametrize("kind", ["normal", "heavy", "bimodal", "ties"])
@pytest.mark.parametrize("k", [4, 16])
def test_lloyd_codebook_matches_sklearn_quality(kind, k):
    sk = pytest.importorskip("sklearn.cluster")
    rng = np.random.default_rng(k * 7 + len(kind))
    vals = _samples(kind, 4000, rng).astype(np.float32)
    lo, up, c, it = oc.calibrate_group(vals, k, 0.005)
    assert lo == float(np.quantile(vals, 0.005)) and up == float(np.quantile(vals, 0.995))
    mass = vals[(vals >= lo) & (vals <= up)]
    km = sk.KMeans(n_clusters=k, n_init=3, max_iter=20, random_state=0).fit(mass.reshape(-1, 1))
    ours, theirs = oc.inertia(mass, c), oc.inertia(mass, km.cluster_centers_.ravel())
    assert np.all(np.diff(c) >= 0) and it <= 20
    assert ours <= theirs * (1 + 1e-9) + 1e-12, (ours, theirs)     # the exact optimum, then Lloyd


def test_fewer_samples_than_levels_pad_with_zeros():
    c, it = oc.kmeans_1d(np.array([3.0, -1.0], np.float32), 4)
    np.testing.assert_array_equal(c, [-1.0, 0.0, 0.0, 3.0])
    c, _ = oc.kmeans_1d(np.array([], np.float32), 4)
    np.testing.assert_array_equal(c, np.zeros(4))
