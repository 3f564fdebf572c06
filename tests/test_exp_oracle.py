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


def test_simd_exp_matches_exp_within_the_reference_bar(oracle):
    """Ops.Exp as restated (the exponential of the decoder's softmax and
    SiLU) is within the reference's own bar against MathF.Exp, 2e-6
    relative (tests/Needle.Tests/KernelTests.cs:35-43), over the range it
    does not clamp."""
    rng = np.random.default_rng(2)
    x = np.concatenate([rng.uniform(-87.0, 88.0, 1_000_000), rng.uniform(-20.0, 0.0, 1_000_000),
                        np.float32(-9.0) + np.float32(2.7) * np.arange(8, dtype=np.float32)]).astype(np.float32)
    got = oracle.exp_simd(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    assert np.all(np.abs(got / ref - 1.0) <= 2e-6)
    # the clamp: below -87.3 the value of exp(-87.3), above 88.7 the overflow to infinity
    low = oracle.exp_simd(np.array([-100.0, -87.3, np.nan], np.float32))
    assert low[0] == low[1] == low[2] > 0
    assert np.isinf(oracle.exp_simd(np.array([89.0], np.float32))[0])


def test_simd_attention_tier_within_the_reference_bar_of_the_scalar_tier(oracle):
    """The AVX2 attention tier the decoder restates stays within the
    reference's tier-to-tier bar of its scalar tier: 3e-5 x peak |output|
    (tests/Needle.Tests/KernelTests.cs:231-236)."""
    import sys, os

    sys.path.insert(0, os.path.dirname(__file__))
    from attention_support import make_case, oracle_out

    lengths = [1, 2, 3, 5, 63, 64, 65, 130, 511, 777, 1024]
    case = make_case(17, lengths, 4)
    simd = oracle_out(oracle, case, lengths, tier="simd")
    scalar = oracle_out(oracle, case, lengths, tier="scalar")
    for r in range(len(lengths)):
        peak = np.abs(scalar[r]).max()
        assert np.all(np.abs(simd[r] - scalar[r]) <= 3e-5 * peak), lengths[r]
