"""KernelTable-signature exports (ndl_kt_*) on the GPU against the
reference's golden vectors and conformance cases, as the reference's own
KernelConformanceTests drive a native kernel slot
(tests/Needle.Tests/Conformance/KernelConformanceTests.cs:1023-1362).

QuantizeInt8 and ArgMaxMasked are bit-exact.  BestProbability is a sum of
exponentials whose order differs from the reference's vector sum: the golden
tolerance applies, and on a long row the result is checked against a
float64 sum (the oracle's sequential fp32 sum is itself only good to about
sqrt(n) ulps there)."""
import numpy as np
import pytest

from test_oracle_golden import _argmax_masked_brute, _mask_case

pytestmark = pytest.mark.gpu


def _lib():
    from needle_cs_b200._native import lib
    return lib()


def _quantize(x):
    x = np.ascontiguousarray(x, np.float32)
    q = np.empty(x.size, np.int8)
    s = _lib().ndl_kt_quantize_int8(x.ctypes.data, x.size, q.ctypes.data)
    return q, np.float32(s)


def test_kt_quantize_int8_golden_and_random(pkg, cuda, oracle, golden):
    fx = golden["fixtures"]
    g = golden["csharp_asserts"]["QuantizeInt8Golden"]
    q, s = _quantize(g["input"])
    assert s == np.float32(fx["QuantizeInt8_scale_neg4_0_4"]) and list(q) == g["bytes"]
    q, s = _quantize([127.0, 0.5, 2.5, -0.5, -2.5, 1.5])  # round half to even
    assert s == 1.0 and list(q) == [127, 0, 2, 0, -2, 2]
    rng = oracle.XorShift64(0x5151)
    for n in (1, 7, 48, 512, 2048, 8192):
        x = rng.fill_edges(n, 3.0)
        q, s = _quantize(x)
        qr, sr = oracle.quantize_int8(x)
        assert s == sr and np.array_equal(q, qr), n
    q, s = _quantize(np.zeros(64, np.float32))  # zero row: scale 1
    assert s == 1.0 and not q.any()


def test_kt_argmax_masked_golden_and_cases(pkg, cuda, oracle, golden):
    lib = _lib()
    fx = golden["fixtures"]
    g = golden["csharp_asserts"]["ArgMaxMaskedGolden"]
    x = np.arange(64, dtype=np.float32)
    for mask, want in ((g["mask_single"], fx["ArgMaxMasked_single_bit_word1_bit5"]), (g["mask_empty"], -1)):
        m = np.ascontiguousarray(mask, np.uint32)
        assert lib.ndl_kt_argmax_masked(x.ctypes.data, m.ctypes.data, m.size, 64) == want
    full = np.ascontiguousarray(g["mask_full"], np.uint32)
    ties = np.full(64, 2.0, np.float32)
    assert lib.ndl_kt_argmax_masked(ties.ctypes.data, full.ctypes.data, full.size, 64) == g["expected_tie"]
    c = golden["csharp_asserts"]["ArgMaxMaskedCases"]
    for length, pattern in c["cases"]:
        x, mask, words = _mask_case(oracle, c["seed"], length, pattern, c["fill_scale"])
        m = np.ascontiguousarray(mask if words else np.zeros(1, np.uint32), np.uint32)
        got = lib.ndl_kt_argmax_masked(x.ctypes.data, m.ctypes.data, words, length)
        assert got == _argmax_masked_brute(x, mask, words, length), (length, pattern)


def test_kt_best_probability(pkg, cuda, oracle, golden):
    lib = _lib()
    fx = golden["fixtures"]
    v = np.float32([1, 2, 3])
    assert abs(lib.ndl_kt_best_probability(v.ctypes.data, 3, 3.0) - fx["BestProbability_1_2_3"]) <= 1e-6
    g = golden["csharp_asserts"]["BestProbabilityGolden"]
    vals = np.ascontiguousarray(g["values"], np.float32)
    assert abs(lib.ndl_kt_best_probability(vals.ctypes.data, vals.size, g["best"]) - g["expected"]) <= g["tol"]
    rng = np.random.default_rng(4)
    x = rng.normal(0, 3, 51865).astype(np.float32)
    best = float(x.max())
    got = lib.ndl_kt_best_probability(x.ctypes.data, x.size, best)
    ref64 = 1.0 / np.exp(x.astype(np.float64) - best).sum()
    assert abs(got - ref64) <= 4e-6 * ref64
    assert abs(got - oracle.best_probability(x, best)) <= 2e-4 * ref64
