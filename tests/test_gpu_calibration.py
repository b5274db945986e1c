"""GPU parity: hx_calib_rows against the calibration oracle. The band is
bit-exact with numpy's quantile (as float32); the centres equal the oracle's
Lloyd iterations within float rounding of the prefix sums."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import np16
from oracle import calibrate as oc

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [1, 3, 17, 300, 4096, 40000])
@pytest.mark.parametrize("k,pct", [(4, 0.025), (16, 0.005)])
def test_calib_rows_match_oracle(n, k, pct):
    from kvquant.calibration import calibrate_rows
    rng = np.random.default_rng(n + k)
    rows = [rng.standard_normal(n) * rng.uniform(0.1, 10), rng.standard_t(3, n),
            np.round(rng.standard_normal(n) * 3) / 3, np.full(n, 1.5),
            np.concatenate([rng.normal(-3, 0.3, n // 2), rng.normal(4, 1, n - n // 2)])]
    x = np.stack(rows).astype(np.float32)
    lo, up, c, its = calibrate_rows(torch.from_numpy(x).cuda(), k, pct)
    lo, up, c, its = np16(lo), np16(up), np16(c), np16(its)
    for r in range(x.shape[0]):
        rlo, rup, rc, rit = oc.calibrate_group(x[r], k, pct)
        assert lo[r] == np.float32(rlo) and up[r] == np.float32(rup)
        np.testing.assert_allclose(c[r], rc.astype(np.float32), rtol=2e-6, atol=1e-6)
        assert abs(int(its[r]) - rit) <= 1


def test_calibrate_keys_and_values_shapes_and_bands():
    """The reference's grouping: K per (head, channel) over tokens, V per
    (head, position) over prompts x channels."""
    from kvquant.calibration import CalibrationConfig, calibrate_keys, calibrate_values
    g = torch.Generator(device="cuda").manual_seed(5)
    K = torch.randn((512, 2, 8), generator=g, device="cuda") * 3
    V = torch.randn((4, 64, 2, 8), generator=g, device="cuda")
    cfg = CalibrationConfig(num_bits=2, outlier_pct=0.01)
    ks, vs = calibrate_keys(K, cfg), calibrate_values(V, cfg)
    assert ks.poles.shape == (2, 8, 4) and ks.upper_threshold.shape == (2, 8)
    assert vs.poles.shape == (2, 64, 4) and vs.lower_threshold.shape == (2, 64)
    Kn, Vn = np16(K), np16(V)
    lo, up = oc.band(Kn[:, 1, 5], 0.01)
    assert float(ks.lower_threshold[1, 5]) == np.float32(lo) and float(ks.upper_threshold[1, 5]) == np.float32(up)
    lo, up = oc.band(Vn[:, 33, 1, :].reshape(-1), 0.01)
    assert float(vs.lower_threshold[1, 33]) == np.float32(lo) and float(vs.upper_threshold[1, 33]) == np.float32(up)
    _, _, rc, _ = oc.calibrate_group(Vn[:, 33, 1, :].reshape(-1), 4, 0.01)
    np.testing.assert_allclose(np16(vs.poles[1, 33]), rc.astype(np.float32), rtol=2e-6, atol=1e-6)
