"""The oracle's float exponential (MathF.Exp restated from the mathematics,
oracle/needle_oracle.c exp_rn) against an independent computation: numpy's
double-precision exp rounded to float.  Both are the correctly rounded float
exp except within a hair of a rounding midpoint, so they agree on every
sampled input but a rare few, and never by more than one ulp."""
import numpy as np


def _inputs():
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.uniform(-104.0, 89.0, 1_500_000),
        rng.uniform(-20.0, 0.0, 1_500_000),  # the softmax range
        rng.normal(0.0, 4.0, 500_000),       # SiLU gates
        [0.0, -0.0, 1.0, -1.0, 88.7, 88.73, 89.0, -87.3, -103.0, -103.97, -104.0, 1e-30, -1e-30],
    ]).astype(np.float32)
    return x[(x >= -104.0) & (x <= 89.0)]


def test_exp_matches_double_exp_rounded(oracle):
    x = _inputs()
    got = oracle.exp_rn(x)
    with np.errstate(over="ignore"):
        ref = np.exp(x.astype(np.float64)).astype(np.float32)
    diff = got != ref
    assert int(diff.sum()) <= 3, int(diff.sum())
    if diff.any():
        a = got[diff].view(np.int32).astype(np.int64)
        b = ref[diff].view(np.int32).astype(np.int64)
        assert np.all(np.abs(a - b) <= 1)


def test_exp_special_values(oracle):
    x = np.array([np.nan, np.inf, -np.inf, 100.0, -200.0, 0.0], np.float32)
    y = oracle.exp_rn(x)
    assert np.isnan(y[0]) and y[1] == np.inf and y[2] == 0.0 and y[3] == np.inf and y[4] == 0.0 and y[5] == 1.0
