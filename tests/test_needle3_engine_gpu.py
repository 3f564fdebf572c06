"""The Needle-3 decode step through ndl_forward_batch on a loaded archive
(ndl_engine_create_model), against the oracle's scalar chain of
EngineCore.ForwardBatch with RunLayerBatch (src/Needle/Engine.cs:2303-2596):
embedding, hyper-connections (phi matmuls, gates, Mix4, Sinkhorn), Engram at
its site layer, attention with 3-tap convs, per-head norms, RoPE, an int8 K/V
cache per slot, grouped heads and a sliding window on the local layer, the
gated output and PostNormAdd, the Kronecker MLP, CombineDiff4x4 and the tied
head.

Bar: every logit bit-identical to the oracle's (both sides take the scalar
tier's operations one rounding at a time, MathF.Exp included), for a prefill
batch mixing runs of several rows with single rows, then decode steps past
the sliding window, a slot reset and refill, and greedy sampling.
"""
import numpy as np
import pytest

from cact_support import needle3_decoder_archive
from needle3_support import oracle_for

pytestmark = pytest.mark.gpu

SLOTS, CAPACITY = 6, 32


def _oracle_batch(o, tokens, row_slots, heads):
    """ForwardBatch with runs on the oracle: wave w feeds the w-th row of every
    run (the reference's run semantics), heads collected in the caller's order."""
    wave, index = [], []
    for r, s in enumerate(row_slots):
        wave.append(wave[-1] + 1 if r > 0 and row_slots[r - 1] == s else 0)
    out = {}
    for w in range(max(wave) + 1):
        rows = [r for r in range(len(tokens)) if wave[r] == w]
        hs = [h for h in heads if wave[h] == w]
        lg = o.forward([tokens[r] for r in rows], [row_slots[r] for r in rows], [rows.index(h) for h in hs])
        for h, row in zip(hs, lg):
            out[h] = row
    return np.stack([out[h] for h in heads])


def _engine_logits(eng, heads):
    return np.stack([eng.batch_logits_row(i) for i in range(len(heads))])


@pytest.fixture(scope="module")
def needle3(pkg):
    import importlib

    cact = importlib.import_module("needle_cs_b200.model")
    engine = importlib.import_module("needle_cs_b200.engine")
    a = needle3_decoder_archive(seed=3)
    m = cact.Model(a.build(), device=0)
    eng = engine.BatchedEngine.from_model(m, slots=SLOTS, context_length=CAPACITY, chunk_size=16, max_heads=16)
    yield a, m, eng
    eng.close()
    m.close()


def test_needle3_step_matches_the_scalar_chain(needle3, oracle):
    a, m, eng = needle3
    o = oracle_for(a, m, SLOTS, CAPACITY)
    rng = np.random.default_rng(7)
    V = m.info["vocab"]
    assert eng.vocab_size == V
    # prefill: runs of 5, 3 and 2 rows and a single row; heads at each run's last row
    row_slots = [0] * 5 + [1] * 3 + [2] + [4] * 2
    tokens = [int(t) for t in rng.integers(0, V, len(row_slots))]
    heads = [4, 7, 8, 10]
    eng.forward_batch(tokens, row_slots, heads)
    want = _oracle_batch(o, tokens, row_slots, heads)
    got = _engine_logits(eng, heads)
    assert np.isfinite(want).all() and np.abs(want).max() > 1.0
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), np.abs(got - want).max()
    assert [eng.slot_length(s) for s in range(SLOTS)] == [5, 3, 1, 0, 2, 0]
    # decode steps, one row per slot, past the local layer's window of 8
    live = [0, 1, 2, 4]
    for step in range(14):
        tokens = [int(t) for t in rng.integers(0, V, len(live))]
        eng.forward_batch(tokens, live, list(range(len(live))))
        want = o.forward(tokens, live, list(range(len(live))))
        got = _engine_logits(eng, live)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (step, np.abs(got - want).max())
    ids = eng.sample_argmax()
    assert list(ids) == [int(i) for i in want.argmax(axis=1)]
    # a reset slot starts over; the others keep their state
    eng.reset_slot(1)
    o.reset_slot(1)
    tokens = [int(t) for t in rng.integers(0, V, 4)]
    row_slots = [1, 1, 1, 3]
    eng.forward_batch(tokens, row_slots, [2, 3])
    want = _oracle_batch(o, tokens, row_slots, [2, 3])
    assert np.array_equal(_engine_logits(eng, [2, 3]).view(np.uint32), want.view(np.uint32))
    # greedy decode of three slots for a few steps, ids fed back
    live = [0, 1, 3]
    ids = [int(i) for i in want.argmax(axis=1)][:1] + [5, 9]
    for step in range(4):
        eng.forward_batch(ids, live, [0, 1, 2])
        got_ids = [int(i) for i in eng.sample_argmax()]
        want_ids = [int(i) for i in o.forward(ids, live, [0, 1, 2]).argmax(axis=1)]
        assert got_ids == want_ids
        ids = got_ids


def test_needle3_mark_rewind_and_primed_prefix(needle3, oracle):
    """MarkSlot / RewindSlot restore the histories, previous tokens and length;
    the primed-prefix blob carries the reference's state section (conv and
    Engram histories, previous tokens) and the marked cache positions, byte
    for byte the oracle's; a slot imported from it decodes exactly as the
    slot it came from."""
    a, m, eng = needle3
    for s in range(SLOTS):
        eng.reset_slot(s)
    o = oracle_for(a, m, SLOTS, CAPACITY)
    rng = np.random.default_rng(11)
    V = m.info["vocab"]
    prompt = [int(t) for t in rng.integers(0, V, 6)]
    eng.forward_batch(prompt, [0] * 6, [5])
    _oracle_batch(o, prompt, [0] * 6, [5])
    eng.mark_slot(0)
    o.mark(0)
    for t in rng.integers(0, V, 3):  # decode past the mark, then back
        eng.forward_batch([int(t)], [0], [0])
        o.forward([int(t)], [0], [0])
    eng.rewind_slot(0)
    o.rewind(0)
    assert eng.slot_length(0) == 6
    blob = eng.export_prefix(0)
    want = o.prefix_blob(0)
    assert len(blob) == len(want) == eng.prefix_bytes(0)
    assert blob == want
    eng.import_prefix(3, blob)
    assert eng.slot_length(3) == 6
    o.reset_slot(3)
    o.keys[3], o.values[3], o.kscale[3], o.vscale[3] = o.keys[0], o.values[0], o.kscale[0], o.vscale[0]
    for name in ("qhist", "khist", "vhist", "ehist", "prev"):
        getattr(o, name)[3] = getattr(o, name)[0]
    o.length[3] = 6
    for step in range(3):
        tok = [int(t) for t in rng.integers(0, V, 1)] * 2
        eng.forward_batch(tok, [0, 3], [0, 1])
        got = _engine_logits(eng, [0, 1])
        want = o.forward(tok, [0, 3], [0, 1])
        assert np.array_equal(got[0].view(np.uint32), got[1].view(np.uint32))  # the import decodes as the source
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), step


def test_needle3_engine_limits(needle3):
    from needle_cs_b200._native import NeedleError

    _, m, eng = needle3
    eng.reset_slot(5)
    with pytest.raises(NeedleError) as e:
        eng.feed_slot(5, list(range(CAPACITY + 1)))
    assert e.value.status == 3
    with pytest.raises(NeedleError) as e:  # rows of one slot must be consecutive
        eng.forward_batch([1, 2, 3], [5, 0, 5], [])
    assert e.value.status == 100
    for op in (lambda: eng.copy_slot(1, 0), lambda: eng.share_prefix(1, 0), lambda: eng.slot_page(0, 0)):
        with pytest.raises(NeedleError) as e:
            op()
        assert e.value.status == 105
