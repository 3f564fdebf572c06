"""Grammar-constrained sparse head on the GPU: Engine.LogitsForBatchRow
(src/Needle/Engine.cs:2683-2700) and ArgMaxSparse
(src/Needle/NeedleSession.cs:984-995) through ndl_logits_sparse.

Bars: every sparse logit equals the dense head's logit of that row at that id
bit for bit, also after a step that computed no dense head; the pick equals
the oracle's ArgMaxSparse on the same values exactly and its probability is
within 1e-6 relative (the sum order differs); malformed requests fail with
NDL_ERR_INVALID_ARG (100) and leave the engine usable.
"""
import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SMALL = dict(layers=2, dim=128, heads=2, head_dim=64, ffn=256, vocab=1000, seed=7)
SLOTS = 8
LENGTHS = [1, 9, 30, 64, 65, 100, 130, 200]


def _engine(eng_mod):
    return eng_mod.BatchedEngine(eng_mod.SyntheticDecoder(**SMALL), slots=SLOTS, context_length=256, chunk_size=16)


@pytest.fixture(scope="module")
def engines(pkg, cuda):
    eng_mod = importlib.import_module("needle_cs_b200.engine")
    dense, bare = _engine(eng_mod), _engine(eng_mod)
    for e in (dense, bare):
        for s, n in enumerate(LENGTHS):
            e.fill_synthetic(s, n, 3, 70 + s)
    tokens = [11 + 97 * s for s in range(SLOTS)]
    rows = list(range(SLOTS))
    dense.forward_batch(tokens, rows, rows)  # a dense head on every row
    bare.forward_batch(tokens, rows, [])  # no dense head at all
    dense_logits = np.stack([dense.batch_logits_row(r).copy() for r in rows])
    yield dense, bare, dense_logits
    dense.close()
    bare.close()


def _lists(rng, vocab):
    return [
        rng.choice(vocab, 40, replace=False),  # a typical grammar set
        np.array([vocab - 1]),  # one id, the last row of the head
        np.array([], np.int32),  # nothing allowed
        rng.integers(0, vocab, 300),  # repeats, unsorted
        np.arange(0, vocab, 3),  # a long strided run
        np.array([5, 4, 3, 2, 1, 0]),  # descending
        rng.choice(vocab, 256, replace=False),
        np.arange(vocab),  # everything
    ]


@pytest.mark.parametrize("which", ["dense", "bare"])
def test_sparse_logits_equal_dense(engines, which):
    dense, bare, dense_logits = engines
    eng = dense if which == "dense" else bare
    V = SMALL["vocab"]
    lists = _lists(np.random.default_rng(5), V)
    rows = [3, 0, 7, 5, 1, 2, 6, 4]
    vals, _, _ = eng.logits_sparse(rows, lists)
    for r, ids, v in zip(rows, lists, vals):
        want = dense_logits[r][np.asarray(ids, np.int64)]
        assert v.dtype == np.float32 and v.shape == want.shape
        assert np.array_equal(v.view(np.uint32), want.view(np.uint32)), (r, ids[:8])


def test_sparse_pick_matches_oracle(engines, oracle):
    _, bare, dense_logits = engines
    V = SMALL["vocab"]
    rng = np.random.default_rng(11)
    lists = _lists(rng, V)
    # plant ties: a list holding the same id twice and an id of equal value
    top = int(np.argmax(dense_logits[2]))
    lists[0] = np.array([17, top, 23, top])
    rows = [2, 2, 4, 0, 6, 1, 3, 7]
    vals, picks, probs = bare.logits_sparse(rows, lists, pick=True, with_probs=True)
    for r, ids, v, got, p in zip(rows, lists, vals, picks, probs):
        want, pw = oracle.argmax_sparse(v, ids)
        assert got == want, (r, got, want)
        if want < 0:
            assert p == 0.0
        else:
            assert abs(p - pw) <= 1e-6 * pw, (p, pw)
    assert picks[2] == -1  # the empty list


def test_sparse_pick_without_values(engines, oracle):
    _, bare, dense_logits = engines
    lists = [np.arange(0, 1000, 7), np.array([9, 8, 7])]
    _, picks, probs = bare.logits_sparse([5, 1], lists, values=False, pick=True)
    assert probs is None
    for r, ids, got in zip([5, 1], lists, picks):
        want, _ = oracle.argmax_sparse(dense_logits[r][ids], ids)
        assert got == want


def test_sparse_rejects_bad_requests(engines):
    from needle_cs_b200 import NeedleError

    _, bare, dense_logits = engines
    for rows, lists in [([SLOTS], [np.array([1])]),  # row outside the last step
                        ([-1], [np.array([1])]),
                        ([0], [np.array([SMALL["vocab"]])]),  # id outside the vocabulary
                        ([0], [np.array([-1])])]:
        with pytest.raises(NeedleError) as e:
            bare.logits_sparse(rows, lists)
        assert e.value.status == 100
    vals, _, _ = bare.logits_sparse([0], [np.array([1, 2])])  # still usable
    assert np.array_equal(vals[0], dense_logits[0][[1, 2]])


def test_sparse_many_requests(engines):
    """As many requests as the engine has head rows, every one on its own list."""
    dense, _, dense_logits = engines
    n = dense.max_heads  # chunk_size 16
    rng = np.random.default_rng(2)
    rows = rng.integers(0, SLOTS, n)
    lists = [rng.integers(0, SMALL["vocab"], int(rng.integers(0, 60))) for _ in range(n)]
    vals, picks, _ = dense.logits_sparse(rows, lists, pick=True)
    for r, ids, v, got in zip(rows, lists, vals, picks):
        assert np.array_equal(v, dense_logits[r][ids])
        if ids.size:
            assert got == ids[int(np.argmax(v))]  # argmax returns the first maximum, like ArgMaxSparse
        else:
            assert got == -1
