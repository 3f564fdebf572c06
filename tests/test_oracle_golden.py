"""The CPU oracle against the reference's own golden vectors and literal asserts.

The fixture tests/golden/conformance_golden.json was produced by running the
reference's tools/conformance_fixtures.py golden() (see make_golden.py).
"""
import math

import numpy as np
import pytest


def f32(x):
    return float(np.float32(x))


def test_softmax_fixtures(oracle, golden):
    fx = golden["fixtures"]
    assert np.array_equal(oracle.softmax([0, 0, 0]), np.float32(fx["Softmax_0_0_0"]))
    assert np.array_equal(oracle.softmax([1, 2, 3]), np.float32(fx["Softmax_1_2_3"]))
    g = golden["csharp_asserts"]["SoftmaxGolden"]
    out = oracle.softmax(g["input"])
    assert np.all(np.abs(out - np.float32(g["expected"])) <= g["tol"])
    assert np.all(np.abs(oracle.softmax(g["uniform_input"]) - g["uniform_expected"]) <= g["tol"])


def test_softmax_tie_first_wins(oracle, golden):
    # the argmax over a tied softmax picks the first index
    assert golden["fixtures"]["Softmax_tie_first_wins"] == 0
    x = np.float32([2.0, 2.0, 1.0])
    assert oracle.lib().ndo_argmax(oracle.ptr(x), 3) == 0


def test_best_probability(oracle, golden):
    fx = golden["fixtures"]
    assert oracle.best_probability([1, 2, 3], 3.0) == np.float32(fx["BestProbability_1_2_3"])
    g = golden["csharp_asserts"]["BestProbabilityGolden"]
    assert abs(oracle.best_probability(g["values"], g["best"]) - g["expected"]) <= g["tol"]
    assert oracle.best_probability([0.7], 0.7) == 1.0


def test_argmax_sparse(oracle, golden):
    """ArgMaxSparse (NeedleSession.cs:984-995): list order decides ties, the
    probability is BestProbability over the list (pinned by its golden)."""
    fx = golden["fixtures"]
    best, p = oracle.argmax_sparse([1, 2, 3], [40, 7, 12])
    assert best == 12 and p == np.float32(fx["BestProbability_1_2_3"])
    assert oracle.argmax_sparse([5, 9, 9, 1], [3, 8, 2, 9])[0] == 8  # first listed maximum, not the lowest id
    assert oracle.argmax_sparse([], []) == (-1, 0.0)
    assert oracle.argmax_sparse([-np.inf, -np.inf], [1, 2]) == (-1, 0.0)  # nothing above -inf
    assert oracle.argmax_sparse([np.nan, 2.0], [4, 6])[0] == 6  # NaN never wins


def test_rms_unit(oracle, golden):
    x = np.float32([3.0, 4.0])
    inv = oracle.lib().ndo_inverse_rms(oracle.ptr(x), 2)
    got = np.float32([x[0] * inv, x[1] * inv])
    assert np.array_equal(got, np.float32(golden["fixtures"]["RmsUnit_3_4"]))
    # the synthetic RMSNorm with unit weight is the same expression
    assert np.array_equal(oracle.rms_norm(x[None, :], np.ones(2, np.float32))[0], got)


def test_quantize_int8_golden(oracle, golden):
    fx = golden["fixtures"]
    g = golden["csharp_asserts"]["QuantizeInt8Golden"]
    q, s = oracle.quantize_int8(g["input"])
    assert s == np.float32(fx["QuantizeInt8_scale_neg4_0_4"])
    assert abs(s - g["scale"]) <= g["scale_tol"]
    assert list(q[:3]) == fx["QuantizeInt8_bytes_neg4_0_4"]
    assert list(q) == g["bytes"]


def test_quantize_round_half_even(oracle, golden):
    # FakeA8 ties: 0.5 -> 0 and 2.5 -> 2 with a unit scale (peak 127)
    fx = golden["fixtures"]
    q, s = oracle.quantize_int8([127.0, 0.5, 2.5, -0.5, -2.5, 1.5])
    assert s == 1.0
    assert q[1] == fx["FakeA8_tie_0_5"] and q[2] == fx["FakeA8_tie_2_5"]
    assert list(q[3:]) == [0, -2, 2]


def test_argmax_masked_golden(oracle, golden):
    fx = golden["fixtures"]
    g = golden["csharp_asserts"]["ArgMaxMaskedGolden"]
    x = np.arange(64, dtype=np.float32)
    assert oracle.argmax_masked(x, g["mask_single"], 64) == fx["ArgMaxMasked_single_bit_word1_bit5"] == 37
    assert oracle.argmax_masked(x, g["mask_empty"], 64) == fx["ArgMaxMasked_empty"] == -1
    assert oracle.argmax_masked(np.full(64, 2.0, np.float32), g["mask_full"], 64) == g["expected_tie"]


def _mask_case(oracle, seed, length, pattern, scale):
    """MaskedConformance.RunCase inputs (KernelConformanceTests.cs:1259-1285)."""
    words = (length + 31) // 32
    rng = oracle.XorShift64(seed)
    x = rng.fill_edges(max(length, 1), scale)
    mask = np.zeros(max(words, 1), np.uint32)
    for w in range(words):
        mask[w] = 0 if pattern == 0 else 0xFFFFFFFF if pattern == 1 else (rng.next() & 0xFFFFFFFF)
    if pattern == 2 and words > 0:
        mask[0] = 0
    if length % 32 != 0 and words > 0 and pattern == 1:
        mask[words - 1] &= 0xFFFFFFFF >> (32 - length % 32)
    if pattern == 3:
        x[:length] = 1.0
    return x, mask[:words] if words else mask[:0], words


def _argmax_masked_brute(x, mask, words, length):
    best, peak = -1, -math.inf
    for w in range(words):
        for b in range(32):
            if mask[w] >> b & 1:
                i = w * 32 + b
                if i < length and x[i] > peak:
                    peak, best = x[i], i
    return best


def test_argmax_masked_conformance_cases(oracle, golden):
    g = golden["csharp_asserts"]["ArgMaxMaskedCases"]
    for length, pattern in g["cases"]:
        x, mask, words = _mask_case(oracle, g["seed"], length, pattern, g["fill_scale"])
        expected = _argmax_masked_brute(x, mask, words, length)
        got = oracle.lib().ndo_argmax_masked(oracle.ptr(x), oracle.ptr(mask) if words else None, words, length)
        assert got == expected, (length, pattern)


def test_dot_golden(oracle, golden):
    a = np.arange(1, 9, dtype=np.int8)
    b = np.arange(8, 0, -1, dtype=np.int8)
    assert int(np.dot(a.astype(np.int32), b.astype(np.int32))) == golden["fixtures"]["Dot_1to8_8to1"] == 120
    # the int8 dot inside the I8G32 matmul: one row, one 32-group
    w = np.zeros((1, 32), np.int8)
    q = np.zeros((1, 32), np.int8)
    w[0, :8], q[0, :8] = a, b
    sw = np.array([[0x3C00]], np.uint16)  # fp16 1.0
    y, acc = oracle.matmul_i8g32(q, [1.0], w, sw, want_acc=True)
    assert acc[0, 0, 0] == 120 and y[0, 0] == 120.0


def test_half_decode_matches_ieee_for_finite(oracle):
    bits = np.arange(0x10000, dtype=np.uint16)
    finite = (bits & 0x7C00) != 0x7C00
    ref = bits.view(np.float16).astype(np.float32)
    got = np.array([oracle.lib().ndo_half_to_single(int(b)) for b in bits[finite]], np.float32)
    assert np.array_equal(got, ref[finite])
    assert oracle.lib().ndo_half_to_single(0x7C00) == 65536.0  # the reference's no-Inf decode


def test_topk_logsoftmax_against_float64(oracle):
    rng = np.random.default_rng(7)
    x = rng.normal(size=51865).astype(np.float32)
    x[100] = x[200] = np.float32(9.0)  # tie -> lower index first
    idx, lp, pr = oracle.topk_logsoftmax(x, 3)
    order = sorted(range(len(x)), key=lambda i: (-x[i], i))[:3]
    assert list(idx) == order
    assert idx[0] == 100 and idx[1] == 200
    shift = np.float64(x.max()) + np.log(np.exp(x.astype(np.float64) - x.max()).sum())
    assert np.allclose(lp, x[idx] - shift, atol=1e-5)
    assert np.allclose(pr, np.exp(lp), rtol=1e-6)
    idx2, _, _ = oracle.topk_logsoftmax(x, 3, mask_special_023=True)
    assert not ({0, 2, 3} & set(idx2.tolist()))


def test_merge_partials_against_float64(oracle, golden):
    """MergePartialsConformance (KernelConformanceTests.cs:494-560)."""
    g = golden["csharp_asserts"]["MergePartialsCases"]
    stride, peak_off = 6 * 64 + 16, 6 * 64
    for count, heads in g["cases"]:
        rng = oracle.XorShift64(count * 31 + heads * 7 + 0xF001)
        partials = np.zeros(count * stride, np.float32)
        for c in range(count):
            chunk = rng.fill_edges(heads * 64, 2.0)
            partials[c * stride:c * stride + heads * 64] = chunk[:heads * 64]
            for h in range(heads):
                partials[c * stride + peak_off + h] = rng.next_float(2.0)
                partials[c * stride + peak_off + 8 + h] = 0.5 + abs(rng.next_float(2.0))
        got = oracle.merge_partials(partials, count, heads, stride, peak_off)
        for h in range(heads):
            peaks = np.float64([partials[c * stride + peak_off + h] for c in range(count)])
            sums = np.float64([partials[c * stride + peak_off + 8 + h] for c in range(count)])
            wts = np.exp(peaks - peaks.max())
            total = (wts * sums).sum()
            for d in range(64):
                num = sum(wts[c] * np.float64(partials[c * stride + h * 64 + d]) for c in range(count))
                assert abs(got[h * 64 + d] - num / total) <= g["tol"] * max(1.0, abs(num / total)) + 1e-6


def test_attention_tile_cases_probabilities(oracle, golden):
    """AttentionTileConformance inputs; the oracle's captured probabilities
    sum to one and its output equals a float64 evaluation within the
    reference tolerance (5e-5 * peak)."""
    g = golden["csharp_asserts"]["AttentionTileCases"]
    P = g["positions"]
    for kv_heads, heads, first, count, _capture in g["cases"]:
        rng = oracle.XorShift64(kv_heads * 1000 + heads * 100 + first * 7 + count * 13 + 0xBEEF)
        queries = rng.fill_sbyte(heads * 48, False)
        keys = rng.fill_sbyte(P * kv_heads * 48, False)
        values = rng.fill_sbyte(P * kv_heads * 64, False)
        qs = np.float32([0.4 + 0.1 * i for i in range(heads)])
        ks = np.empty(P * kv_heads, np.float32)
        vs = np.empty(P * kv_heads, np.float32)
        for i in range(P * kv_heads):
            ks[i] = np.float32(0.0004) * (1 + rng.next_int(0, 4))
            vs[i] = np.float32(0.003) * (1 + rng.next_int(0, 4))
        kv = kv_heads - 1
        inv = np.float32(0.14433756729740643)
        for h in range(heads):
            probs = np.zeros(P, np.float32)
            out = oracle.attention_head(queries[h * 48:], np.float32(qs[h]), keys[kv * 48:], ks[kv:],
                                        values[kv * 64:], vs[kv:], kv_heads * 48, kv_heads * 64, kv_heads, first,
                                        first + count - 1, 48, 64, inv, probabilities=probs)
            s = np.array([np.float64(np.dot(queries[h * 48:h * 48 + 48].astype(np.int64),
                                            keys[(first + j) * kv_heads * 48 + kv * 48:][:48].astype(np.int64)))
                          * ks[(first + j) * kv_heads + kv] * qs[h] * inv for j in range(count)])
            p = np.exp(s - s.max())
            p /= p.sum()
            ref = sum(p[j] * vs[(first + j) * kv_heads + kv] *
                      values[(first + j) * kv_heads * 64 + kv * 64:][:64].astype(np.float64) for j in range(count))
            peak = np.abs(ref).max()
            assert np.all(np.abs(out - ref) <= 5e-5 * peak + 1e-7)
            assert abs(probs[first:first + count].sum() - 1.0) < 1e-5


def test_i8g32_matches_numpy_int(oracle):
    rng = np.random.default_rng(3)
    m, n, k = 5, 37, 256
    q = rng.integers(-128, 128, (m, k), dtype=np.int8)
    w = rng.integers(-127, 128, (n, k), dtype=np.int8)
    sw = np.float16(rng.uniform(0.001, 0.02, (n, k // 32))).view(np.uint16)
    sa = rng.uniform(0.01, 0.1, m).astype(np.float32)
    y, acc = oracle.matmul_i8g32(q, sa, w, sw, want_acc=True)
    d = np.einsum("tgk,ngk->tng", q.reshape(m, -1, 32).astype(np.int64), w.reshape(n, -1, 32).astype(np.int64))
    assert np.array_equal(acc, d)
    ref = (sw.view(np.float16).astype(np.float64)[None] * sa[:, None, None] * d).sum(-1)
    assert np.allclose(y, ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("bits,cols", [(2, 128), (4, 384), (2, 768)])
def test_cq_gather_row_matches_float(oracle, bits, cols):
    """Quant.GatherRow (DecodeRow, then the scaled Walsh-Hadamard transform
    per group) equals a float64 evaluation with the Sylvester matrix."""
    rng = np.random.default_rng(bits * 1000 + cols)
    rows, groups = 3, cols // 128
    idx = rng.integers(0, 256, (rows, cols * bits // 8), dtype=np.uint8)
    norms = np.float16(rng.uniform(0.2, 2.0, (rows, groups))).view(np.uint16)
    levels = np.linspace(-1.0, 1.0, 16).astype(np.float32)
    h = np.array([[1.0]])
    while h.shape[0] < 128:
        h = np.block([[h, h], [h, -h]])
    for row in range(rows):
        got = oracle.gather_row_cq(idx, norms, levels, bits, row)
        if bits == 2:
            codes = np.stack([(idx[row] >> (2 * p)) & 3 for p in range(4)], 1).reshape(-1)
        else:
            codes = np.stack([idx[row] & 15, idx[row] >> 4], 1).reshape(-1)
        dec = levels[codes].astype(np.float64).reshape(groups, 128) * \
            norms[row].view(np.float16).astype(np.float64)[:, None]
        want = (dec @ h.T * 0.08838834764831845).reshape(-1)
        assert np.allclose(got, want, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("bits,rows,cols,tokens", [(2, 4, 128, 2), (4, 4, 128, 2), (2, 5, 768, 3), (4, 7, 384, 5)])
def test_cq_matmul_matches_dequantized_float(oracle, bits, rows, cols, tokens):
    """Scalar.MatMulRows on ConformanceWeights-style CQ inputs equals a
    float64 evaluation of the same codebook bytes and offsets."""
    import ctypes

    rng = oracle.XorShift64(0x1234)
    count = 4 if bits == 2 else 16
    levels = np.zeros(16, np.float32)
    for i in range(count):
        levels[i] = np.float32((i - (count - 1) / 2) * 0.4) + np.float32(
            (float(np.float32(rng.next() >> 11)) * (1.0 / 9007199254740992.0) - 0.5) * 0.1)
    book = (ctypes.c_ubyte * 256)()
    oracle.lib().ndo_codebook_fill(ctypes.addressof(book), oracle.ptr(levels), count)
    table = np.frombuffer(bytes(book)[64:96], np.uint8)
    byte_scale = np.frombuffer(bytes(book)[96:100], np.float32)[0]
    row_bytes = cols * bits // 8
    fill = oracle.XorShift64(0x1234 ^ 0x5BD1E995)
    idx = fill.fill_bytes(rows * row_bytes, True)[:rows * row_bytes]
    groups = cols // 128
    norms = np.array([oracle.lib().ndo_half_bits(np.float32(0.2 + (fill.next() % 1000) * 0.0018))
                      for _ in range(rows * groups)], np.uint16)
    x = oracle.XorShift64(0x1234 ^ 0x243F6A88).fill_edges(tokens * cols, 3.0)[:tokens * cols]
    stride = (groups + 7) & ~7
    vals = np.zeros(tokens * cols, np.int8)
    sc = np.zeros(tokens * stride, np.float32)
    off = np.zeros(tokens * stride, np.float32)
    oracle.lib().ndo_prepare_cq(oracle.ptr(x), tokens, cols, bits, oracle.ptr(vals), oracle.ptr(sc),
                                oracle.ptr(off), stride)
    y = np.zeros(tokens * rows, np.float32)
    oracle.lib().ndo_matmul_rows_cq(oracle.ptr(idx), oracle.ptr(norms), ctypes.addressof(book), rows, cols, bits,
                                    oracle.ptr(vals), oracle.ptr(sc), oracle.ptr(off), stride, tokens,
                                    oracle.ptr(y), rows, 0, rows)
    for t in range(tokens):
        for n in range(rows):
            total = 0.0
            for g in range(groups):
                xs = vals[(t * groups + g) * 128:][:128].astype(np.int64)
                if bits == 2:
                    p = idx[n * row_bytes + g * 32:][:32]
                    codes = np.concatenate([table[(p >> (2 * s)) & 3] for s in range(4)]).astype(np.int64)
                else:
                    p = idx[n * row_bytes + g * 64:][:64]
                    codes = np.concatenate([table[p[:32] & 15], table[p[:32] >> 4], table[p[32:] & 15],
                                            table[p[32:] >> 4]]).astype(np.int64)
                dot = int((codes * xs).sum())
                f = np.float64(oracle.lib().ndo_half_to_single(int(norms[n * groups + g]))) * byte_scale * \
                    sc[t * stride + g]
                total += f * (dot - off[t * stride + g])
            assert abs(y[t * rows + n] - total) <= 1e-3 * max(1.0, abs(total))
