"""The reference's AttentionTile, MergePartials and HadamardMlp KernelTable
slots (3, 4, 5) on the GPU (Attention.Run / Scalar.AttentionTile,
src/Needle/Blocks.cs:65-84, src/Needle/Scalar.cs:290-321;
Attention.MergePartials, Blocks.cs:750-817; HadamardMlp.Apply,
Blocks.cs:1067-1093).

Bars (the reference's own, KernelTests.cs:231-236): tile outputs within
3e-5 x the peak |output| of the oracle's scalar restatement; probabilities
within 1e-6 absolute.  The split-position mode (peaks and sums set) merged by
MergePartials must give the unsplit tile's result within the same bar.
HadamardMlp: bit-exact (its softmax and SiLU take the correctly rounded
exponential on both sides).  Tile cases follow AttentionTileCases (counts 1, 2, 4, 45;
firsts 0, 13, 41; heads 1, 2, 6; int8 extremes).
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

P = ctypes.c_void_p


class KtTile(ctypes.Structure):
    _fields_ = [("queries", P), ("query_scales", P), ("heads", ctypes.c_int), ("keys", P), ("key_scales", P),
                ("values", P), ("value_scales", P), ("key_stride", ctypes.c_int), ("value_stride", ctypes.c_int),
                ("scale_stride", ctypes.c_int), ("first", ctypes.c_int), ("count", ctypes.c_int), ("scores", P),
                ("output", P), ("probabilities", P), ("probability_stride", ctypes.c_int), ("peaks", P),
                ("sums", P)]


class KtMlpWeights(ctypes.Structure):
    _fields_ = [(n, P) for n in ("d1", "d2", "b2", "d3", "d4", "w1a", "w1b", "w2a", "w2b", "w3a", "w3b", "cond_v",
                                 "cond_u")]


class KtMlpBatch(ctypes.Structure):
    _fields_ = [("weights", P), ("pre_norm", P), ("perm_a", P), ("perm_b", P), ("residual", P),
                ("dim", ctypes.c_int), ("rows", ctypes.c_int), ("cols", ctypes.c_int), ("scale", ctypes.c_float)]


STRIDE, PEAK = 6 * 64 + 16, 6 * 64


def _case(seed, heads, span, extremes=False):
    rng = np.random.default_rng(seed)
    key_stride, value_stride, scale_stride = 56, 72, 2  # padded rows, interleaved scales
    keys = rng.integers(-128, 128, (span, key_stride)).astype(np.int8)
    values = rng.integers(-128, 128, (span, value_stride)).astype(np.int8)
    if extremes:
        keys[::3] = 127
        values[1::3] = -128
    q = rng.integers(-128, 128, (heads, 48)).astype(np.int8)
    qs = rng.uniform(0.01, 0.05, heads).astype(np.float32)
    ks = rng.uniform(0.005, 0.03, span * scale_stride).astype(np.float32)
    vs = rng.uniform(0.005, 0.03, span * scale_stride).astype(np.float32)
    return dict(q=q, qs=qs, keys=keys, values=values, ks=ks, vs=vs, ks_stride=key_stride, vs_stride=value_stride,
                sc_stride=scale_stride)


def _run_tile(lib, c, heads, first, count, partial=False, probs_stride=None):
    out = np.full((heads, 64), 9.0, np.float32)
    scores = np.zeros(max(count, 1) * 8, np.float32)
    probs = np.full(heads * probs_stride, -1.0, np.float32) if probs_stride else None
    peaks = np.zeros(8, np.float32) if partial else None
    sums = np.zeros(8, np.float32) if partial else None
    t = KtTile(c["q"].ctypes.data, c["qs"].ctypes.data, heads, c["keys"].ctypes.data, c["ks"].ctypes.data,
               c["values"].ctypes.data, c["vs"].ctypes.data, c["ks_stride"], c["vs_stride"], c["sc_stride"], first,
               count, scores.ctypes.data, out.ctypes.data, probs.ctypes.data if probs is not None else None,
               probs_stride or 0, peaks.ctypes.data if partial else None, sums.ctypes.data if partial else None)
    lib.ndl_kt_attention_tile(ctypes.byref(t))
    return out, probs, peaks, sums


def _oracle_tile(olib, c, heads, first, count, probs_stride):
    outs = np.zeros((heads, 64), np.float32)
    probs = np.full(heads * probs_stride, -1.0, np.float32)
    scores = np.zeros(count, np.float32)
    for h in range(heads):
        qh = np.ascontiguousarray(c["q"][h])
        olib.ndo_attention_head(qh.ctypes.data, float(c["qs"][h]), c["keys"].ctypes.data, c["ks"].ctypes.data,
                                c["values"].ctypes.data, c["vs"].ctypes.data, c["ks_stride"], c["vs_stride"],
                                c["sc_stride"], first, first + count - 1, 48, 64, 0.14433756729740643,
                                scores.ctypes.data, outs[h].ctypes.data, probs.ctypes.data + h * probs_stride * 4)
    return outs, probs


@pytest.mark.parametrize("heads", [1, 2, 6])
@pytest.mark.parametrize("count,first", [(1, 0), (2, 13), (4, 41), (45, 0), (45, 13), (300, 41)])
def test_attention_tile_matches_oracle(pkg, cuda, oracle, heads, count, first):
    lib, olib = pkg.lib(), oracle.lib()
    c = _case(heads * 1000 + count + first, heads, first + count + 3, extremes=count == 4)
    stride = first + count + 5
    got, gp, _, _ = _run_tile(lib, c, heads, first, count, probs_stride=stride)
    want, wp = _oracle_tile(olib, c, heads, first, count, stride)
    peak = max(float(np.abs(want).max()), 1e-12)
    assert np.abs(got - want).max() <= 3e-5 * peak
    assert np.allclose(gp, wp, atol=1e-6, rtol=0)  # positions outside [first, first + count) stay -1


@pytest.mark.parametrize("heads,count,chunks", [(1, 45, 2), (2, 300, 3), (6, 128, 2), (6, 90, 5)])
def test_split_tiles_merge_to_the_whole(pkg, cuda, oracle, heads, count, chunks):
    lib, olib = pkg.lib(), oracle.lib()
    c = _case(7 * count + chunks, heads, count)
    whole, _, _, _ = _run_tile(lib, c, heads, 0, count)
    bounds = np.linspace(0, count, chunks + 1).astype(int)
    partials = np.zeros(chunks * STRIDE, np.float32)
    for k in range(chunks):
        o, _, pk, sm = _run_tile(lib, c, heads, int(bounds[k]), int(bounds[k + 1] - bounds[k]), partial=True)
        partials[k * STRIDE:k * STRIDE + heads * 64] = o.reshape(-1)
        partials[k * STRIDE + PEAK:k * STRIDE + PEAK + heads] = pk[:heads]
        partials[k * STRIDE + PEAK + 8:k * STRIDE + PEAK + 8 + heads] = sm[:heads]
    merged = np.zeros(heads * 64, np.float32)
    lib.ndl_kt_merge_partials(partials.ctypes.data, chunks, heads, merged.ctypes.data)
    want = np.zeros(heads * 64, np.float32)
    olib.ndo_merge_partials(partials.ctypes.data, chunks, heads, STRIDE, PEAK, want.ctypes.data)
    peak = float(np.abs(whole).max())
    assert np.abs(merged - want).max() <= 1e-6 * peak  # the merge itself
    assert np.abs(merged.reshape(heads, 64) - whole).max() <= 3e-5 * peak  # split == whole


def test_merge_partials_golden_cases(pkg, cuda, oracle, golden):
    """MergePartialsConformance inputs (KernelConformanceTests.cs:494-560)."""
    lib, olib = pkg.lib(), oracle.lib()
    for count, heads in golden["csharp_asserts"]["MergePartialsCases"]["cases"]:
        rng = oracle.XorShift64(count * 31 + heads * 7 + 0xF001)
        partials = np.zeros(count * STRIDE, np.float32)
        for ch in range(count):
            partials[ch * STRIDE:ch * STRIDE + heads * 64] = rng.fill_edges(heads * 64, 2.0)[:heads * 64]
            for h in range(heads):
                partials[ch * STRIDE + PEAK + h] = rng.next_float(2.0)
                partials[ch * STRIDE + PEAK + 8 + h] = 0.5 + abs(rng.next_float(2.0))
        got = np.zeros(heads * 64, np.float32)
        want = np.zeros(heads * 64, np.float32)
        lib.ndl_kt_merge_partials(partials.ctypes.data, count, heads, got.ctypes.data)
        olib.ndo_merge_partials(partials.ctypes.data, count, heads, STRIDE, PEAK, want.ctypes.data)
        assert np.allclose(got, want, rtol=2e-6, atol=1e-6 * max(1.0, float(np.abs(want).max()))), (count, heads)


@pytest.mark.parametrize("dim,rows,cols,perm", [(128, 4, 32, "identity"), (128, 4, 32, "rotated"),
                                                (100, 4, 32, "random"), (768, 32, 32, "random")])
def test_hadamard_mlp_slot(pkg, cuda, oracle, dim, rows, cols, perm):
    """HadamardMlp.Apply (slot 5) against the oracle's scalar restatement
    (HadamardMlp conformance entry: dim 128, rows 4, cols 32, identity and
    rotated permutations; then a ragged and a Needle-3-sized case)."""
    lib, olib = pkg.lib(), oracle.lib()
    rng = np.random.default_rng(6750 + dim + rows)
    width, in_rows = rows * cols, (dim + cols - 1) // cols
    arr = {k: rng.normal(0, s, n).astype(np.float32) for k, s, n in (
        ("d1", 1.0, dim), ("d2", 1.0, width), ("b2", 0.1, width), ("d3", 1.0, width), ("d4", 1.0, dim),
        ("w1a", 0.3, in_rows * rows), ("w1b", 0.2, cols * cols), ("w2a", 0.3, rows * rows),
        ("w2b", 0.2, cols * cols), ("w3a", 0.3, rows * rows), ("w3b", 0.2, cols * cols),
        ("cond_v", 0.1, dim * 8), ("cond_u", 0.1, 8 * width))}
    if perm == "identity":
        pa = pb = np.arange(width, dtype=np.int32)
    elif perm == "rotated":
        pa, pb = np.roll(np.arange(width, dtype=np.int32), 7), np.roll(np.arange(width, dtype=np.int32), -3)
    else:
        pa, pb = rng.permutation(width).astype(np.int32), rng.permutation(width).astype(np.int32)
    pre = rng.uniform(-0.3, 0.3, dim).astype(np.float32)
    res = rng.normal(size=dim).astype(np.float32)
    names = [f[0] for f in KtMlpWeights._fields_]
    w = KtMlpWeights(*[arr[n].ctypes.data for n in names])
    b = KtMlpBatch(ctypes.addressof(w), pre.ctypes.data, pa.ctypes.data, pb.ctypes.data, None, dim, rows, cols, 0.5)
    got = res.copy()
    lib.ndl_kt_hadamard_mlp(ctypes.byref(b), got.ctypes.data, None)
    want = res.copy()
    ptrs = (ctypes.c_void_p * 13)(*[arr[n].ctypes.data for n in names])
    olib.ndo_hadamard_mlp(ptrs, pre.ctypes.data, pa.ctypes.data, pb.ctypes.data, dim, rows, cols, 0.5,
                          want.ctypes.data)
    delta = want - res
    assert np.abs(delta).max() > 1e-3  # the MLP did something
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), np.abs(got - want).max()
