"""The oracle's Needle-3 restatements against independent formulations.

The reference holds no golden vectors for these blocks, so each C
restatement is checked on the CPU against the same mathematics written
differently: a pure-Python hash (EngramHashRowsBatch, Engine.cs:2652-2681),
float64 numpy for the Engram conv and gate (ApplyEngramBatch, :2405-2469),
the batch softmax that the online pools must equal (PoolTokensBatch,
:2598-2650, ConfidenceLogitForSlot, :2702-2738), the Kronecker products as
matrix products (HadamardMlp.Apply, Blocks.cs:1067-1093), and the Sinkhorn
iterations in float64 (Scalar.Sinkhorn4x4, Scalar.cs:361-381).
"""
import ctypes

import numpy as np


def _p(a):
    return a.ctypes.data


def test_engram_hash_matches_python(oracle):
    rng = np.random.default_rng(1)
    slots, heads, engram_slots = 8, 3, 1009
    orders = np.array([2, 3], np.int32)
    row_slots = np.array([3, 3, 3, 5, 1, 1, 6], np.int32)
    tokens = rng.integers(0, 1 << 20, row_slots.size).astype(np.int32)
    slot_length = np.array([4, 0, 9, 1, 7, 2, 0, 3], np.int32)
    slot_prev = rng.integers(0, 1 << 20, (slots, 2)).astype(np.int32)
    tables = orders.size * heads
    got = np.zeros((row_slots.size, tables), np.int32)
    oracle.lib().ndo_engram_hash(_p(tokens), _p(row_slots), row_slots.size, _p(slot_length), _p(slot_prev),
                                 _p(orders), orders.size, heads, engram_slots, _p(got))
    for t in range(row_slots.size):
        rs = t
        while rs > 0 and row_slots[rs - 1] == row_slots[t]:
            rs -= 1
        slot = row_slots[t]
        pos = slot_length[slot] + t - rs
        for o, order in enumerate(orders):
            for h in range(heads):
                table = o * heads + h
                if pos < order - 1:
                    assert got[t, table] == -1
                    continue
                acc = (0x9E3779B9 * (table + 1)) & 0xFFFFFFFF
                for j in range(order):
                    back = t - rs - j
                    tok = int(tokens[rs + back]) if back >= 0 else int(slot_prev[slot, back + 2])
                    acc = ((acc ^ (tok & 0xFFFFFFFF)) * 0x01000193) & 0xFFFFFFFF
                acc ^= acc >> 15
                assert got[t, table] == table * engram_slots + acc % engram_slots, (t, table)


def test_engram_conv_and_gate_match_float64(oracle):
    rng = np.random.default_rng(2)
    slots, dim, dil = 4, 64, 2
    row_slots = np.array([2, 2, 2, 0, 3], np.int32)
    hist = rng.normal(size=(slots, 9, dim)).astype(np.float32)
    values = rng.normal(size=(row_slots.size, dim)).astype(np.float32)
    taps = rng.normal(size=(4, dim)).astype(np.float32)
    out = np.zeros((row_slots.size, dim), np.float32)
    hout = hist.copy()
    oracle.lib().ndo_engram_conv(_p(hist), _p(values), _p(row_slots), row_slots.size, _p(taps), dil, dim, _p(out),
                                 _p(hout))
    for s in (2, 0, 3):
        idx = np.flatnonzero(row_slots == s)
        seq = np.concatenate([hist[s], values[idx]]).astype(np.float64)
        for n, t in enumerate(idx):
            want = sum(taps[j].astype(np.float64) * seq[n + 9 - j * dil] for j in range(4))
            assert np.allclose(out[t], want, rtol=1e-5, atol=1e-5)
        assert np.array_equal(hout[s], seq[len(idx):len(idx) + 9].astype(np.float32))
    assert np.array_equal(hout[1], hist[1])  # a slot outside the batch keeps its history
    x, key, v = (rng.normal(size=dim).astype(np.float32) for _ in range(3))
    res = rng.normal(size=dim).astype(np.float32)
    got = res.copy()
    oracle.lib().ndo_engram_gate(_p(x), _p(key), _p(v), dim, _p(got))
    ua = x / np.sqrt((x.astype(np.float64) ** 2).mean() + 1e-6)
    ub = key / np.sqrt((key.astype(np.float64) ** 2).mean() + 1e-6)
    alpha = 1 / (1 + np.exp(-(ua * ub).sum() / np.sqrt(dim)))
    assert np.allclose(got, res + alpha * v, rtol=1e-5, atol=1e-6)


def test_confidence_pools_equal_the_batch_softmax(oracle):
    """Token by token, the online pools end where a softmax over all scores
    does; the logit follows its float64 definition."""
    rng = np.random.default_rng(3)
    slots, dim, probes, pool_rows, n_tok = 2, 32, 2, 4, 7
    probe_v = rng.normal(size=(pool_rows, dim)).astype(np.float32)
    cell = np.zeros((slots, dim), np.float32)
    pmax = np.full((slots, pool_rows), -np.inf, np.float32)
    psum = np.zeros((slots, pool_rows), np.float32)
    pacc = np.zeros((slots, pool_rows, dim), np.float32)
    streams = rng.normal(size=(n_tok, 4, dim)).astype(np.float32)
    row_slots = np.full(n_tok, 1, np.int32)
    oracle.lib().ndo_conf_pool_update(1, _p(streams), _p(row_slots), n_tok, 1, _p(probe_v), probes, dim, pool_rows,
                                      _p(cell), _p(pmax), _p(psum), _p(pacc), None, None, None, None)
    cells = streams.astype(np.float64).mean(axis=1)
    cells[0] = streams[0, 0]  # the first token of an initial run takes stream 0
    for p in range(probes):
        i = probes + p
        sc = cells @ probe_v[i].astype(np.float64) / np.sqrt(dim)
        w = np.exp(sc - sc.max())
        assert np.isclose(pmax[1, i], sc.max(), rtol=1e-5)
        assert np.isclose(psum[1, i], w.sum(), rtol=1e-5)
        assert np.allclose(pacc[1, i], (w[:, None] * cells).sum(0), rtol=1e-4, atol=1e-5)
    assert np.allclose(cell[1], cells[-1], rtol=1e-6)
    # the logit from finite pools
    psum1 = rng.uniform(1, 3, pool_rows).astype(np.float32)
    pacc1 = rng.normal(size=(pool_rows, dim)).astype(np.float32)
    gain = rng.uniform(0.5, 1.5, pool_rows).astype(np.float32)
    qv = rng.normal(size=(2, dim)).astype(np.float32)
    rb = rng.normal(size=(2, pool_rows)).astype(np.float32)
    proj = rng.normal(size=2 * dim).astype(np.float32)
    pooled = np.zeros((2, dim), np.float32)
    logit = oracle.lib().ndo_conf_logit(_p(psum1), _p(pacc1), pool_rows, dim, _p(gain), _p(qv), _p(rb), 0.3, _p(proj),
                                        2, _p(pooled))
    mean = pacc1.astype(np.float64) / psum1[:, None]
    keys = gain[:, None] * mean / np.sqrt((mean ** 2).mean(1, keepdims=True) + 1e-6)
    want_pooled = []
    for q in range(2):
        wts = keys @ qv[q] / np.sqrt(dim) + rb[q]
        wts = np.exp(wts - wts.max())
        want_pooled.append((wts / wts.sum()) @ keys)
    want_pooled = np.array(want_pooled)
    assert np.allclose(pooled, want_pooled, rtol=1e-4, atol=1e-5)
    assert np.isclose(logit, 0.3 + want_pooled.reshape(-1) @ proj, rtol=1e-4, atol=1e-4)


def test_hadamard_mlp_matches_float64(oracle):
    rng = np.random.default_rng(4)
    dim, rows, cols = 100, 4, 32
    width, in_rows = rows * cols, (dim + cols - 1) // cols
    out_rows = min(rows, (in_rows + 3) // 4 * 4)
    arr = {k: rng.normal(0, s, n).astype(np.float32) for k, s, n in (
        ("d1", 1.0, dim), ("d2", 1.0, width), ("b2", 0.1, width), ("d3", 1.0, width), ("d4", 1.0, dim),
        ("w1a", 0.3, in_rows * rows), ("w1b", 0.2, cols * cols), ("w2a", 0.3, rows * rows),
        ("w2b", 0.2, cols * cols), ("w3a", 0.3, rows * rows), ("w3b", 0.2, cols * cols),
        ("cond_v", 0.1, dim * 8), ("cond_u", 0.1, 8 * width))}
    names = ["d1", "d2", "b2", "d3", "d4", "w1a", "w1b", "w2a", "w2b", "w3a", "w3b", "cond_v", "cond_u"]
    pa, pb = rng.permutation(width).astype(np.int32), rng.permutation(width).astype(np.int32)
    pre = rng.uniform(-0.3, 0.3, dim).astype(np.float32)
    res = rng.normal(size=dim).astype(np.float32)
    got = res.copy()
    ptrs = (ctypes.c_void_p * 13)(*[arr[n].ctypes.data for n in names])
    oracle.lib().ndo_hadamard_mlp(ptrs, _p(pre), _p(pa), _p(pb), dim, rows, cols, 0.5, _p(got))
    a = {k: v.astype(np.float64) for k, v in arr.items()}
    x = res.astype(np.float64)
    norm = (1 + pre) * x / np.sqrt((x ** 2).mean() + 1e-6)
    wl = norm @ a["cond_v"].reshape(dim, 8)
    wl = np.exp(wl - wl.max())
    wl /= wl.sum()
    front = np.zeros(in_rows * cols)
    front[:dim] = norm * a["d1"]

    def kron(z, active, left, right, result_rows):  # result = left^T . z . right
        return (left.reshape(-1, rows)[:active].T @ z.reshape(-1, cols)[:active] @ right.reshape(cols, cols))[
            :result_rows].reshape(-1)

    back = kron(front, in_rows, a["w1a"], a["w1b"], rows)
    cond = 1 + wl @ a["cond_u"].reshape(8, width)
    v = a["d2"] * cond * back[pa] + a["b2"]
    front = v / (1 + np.exp(-v))
    back = kron(front, rows, a["w2a"], a["w2b"], rows)
    front = back[pb] * a["d3"]
    back = kron(front, rows, a["w3a"], a["w3b"], out_rows)
    want = x + 0.5 * back[:dim] * a["d4"]
    assert np.allclose(got, want, rtol=1e-4, atol=1e-4)


def test_sinkhorn_matches_float64_iterations(oracle):
    """20 row-then-column normalisations of exp(logits - row peak): columns
    end at 1 (normalised last), rows near it."""
    rng = np.random.default_rng(5)
    for _ in range(10):
        lg = (rng.normal(size=16) * 2).astype(np.float32)
        r = oracle.sinkhorn4x4(lg).reshape(4, 4)
        w = lg.astype(np.float64).reshape(4, 4)
        w = np.exp(w - w.max(1, keepdims=True))
        for _ in range(20):
            w /= w.sum(1, keepdims=True)
            w /= w.sum(0, keepdims=True)
        assert np.allclose(r, w, rtol=1e-4, atol=1e-6)
        assert np.allclose(r.sum(0), 1, atol=1e-5) and np.allclose(r.sum(1), 1, atol=1e-2)
