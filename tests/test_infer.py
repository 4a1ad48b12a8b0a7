"""Interpolation plan (Interpolation.swift:47-58) on CPU: frame counts and times."""
import numpy as np

from yumelayers_b200.trainer import interpolation_plan


def test_plan_counts_and_endpoints():
    assert interpolation_plan(2.0, 24).size == 48
    assert interpolation_plan(1.02, 25).size == 26  # round(25.5) -> 26
    for bad in ((0.0, 24), (-1.0, 24), (1.0, 0), (float("nan"), 24)):
        assert interpolation_plan(*bad).size == 2
    t = interpolation_plan(0.5, 10)
    assert t.size == 5 and t[0] == 0.0 and t[-1] == 1.0
    np.testing.assert_allclose(np.diff(t), 0.25, rtol=0, atol=1e-7)
