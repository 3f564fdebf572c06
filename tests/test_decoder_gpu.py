"""Batched decode step on the GPU against the CPU oracle.

Mirrors the reference's BatchedDecodeTests (tests/Needle.Tests/
BatchedDecodeTests.cs): batched logits against a single-row evaluation, for
single tokens, prefill runs and reordered rows; plus paged-KV contents and
slot rewind.  Bars: synthetic prefix KV and the K/V a step writes
bit-exact; logits bit-identical to the oracle's (every kernel of the step
keeps the reference's rounding order), so the argmax is the oracle's too;
batch-invariant rows bit-identical whatever the batch composition.
"""
import numpy as np
import pytest

from decoder_support import oracle_decoder, prefix_kv, read_slot_kv, top2_margin

pytestmark = pytest.mark.gpu

SMALL = dict(layers=2, dim=128, heads=2, head_dim=64, ffn=256, vocab=1000, seed=7)
PREFIX = [5, 70, 130, 1]


@pytest.fixture(scope="module")
def small(pkg, cuda):
    import importlib

    eng_mod = importlib.import_module("needle_cs_b200.engine")
    model = eng_mod.SyntheticDecoder(**SMALL)
    eng = eng_mod.BatchedEngine(model, slots=6, context_length=256, chunk_size=16)
    yield eng
    eng.close()


def _fresh(eng, seed=3):
    for s in range(eng.slots):
        eng.reset_slot(s)
    for s, n in enumerate(PREFIX):
        eng.fill_synthetic(s, n, seed, 1000 + s)


def test_prefix_fill_bit_exact(small, ops, oracle):
    _fresh(small)
    dec = oracle_decoder(oracle, small)
    for s, n in enumerate(PREFIX):
        kv = dec.new_kv()
        prefix_kv(ops, oracle, dec, kv, n, 3, 1000 + s)
        got = read_slot_kv(small, s, n)
        for key in ("k", "v", "ks", "vs"):
            assert np.array_equal(got[key], kv[key][:, :n]), (s, key)


def test_decode_step_matches_oracle(small, ops, oracle):
    _fresh(small)
    dec = oracle_decoder(oracle, small)
    tokens = [11, 222, 333, 999]
    small.forward_batch(tokens, [0, 1, 2, 3], [0, 1, 2, 3])
    ids = small.sample_argmax()
    for s, n in enumerate(PREFIX):
        kv = dec.new_kv()
        prefix_kv(ops, oracle, dec, kv, n, 3, 1000 + s)
        ref = dec.row(tokens[s], n, kv)
        got = small.batch_logits_row(s)
        assert np.array_equal(got, ref), f"slot {s}: max err {np.abs(got - ref).max()}"
        assert ids[s] == int(np.argmax(ref)), f"slot {s}: margin {top2_margin(ref)}"
        # the new position's K/V (written by the KV-write epilogue), byte for byte
        new = read_slot_kv(small, s, n + 1)
        for key in ("k", "v", "ks", "vs"):
            assert np.array_equal(new[key][:, n], kv[key][:, n]), (s, key)
        assert small.slot_length(s) == n + 1


def test_prefill_run_then_decode(small, ops, oracle):
    """Consecutive rows of one slot are a causal prefill run (Engine.cs:2303-2350)."""
    _fresh(small)
    dec = oracle_decoder(oracle, small)
    run = [5, 6, 7, 8, 9]
    small.forward_batch(run + [42], [1] * 5 + [3], [4, 5])
    kv1 = dec.new_kv()
    prefix_kv(ops, oracle, dec, kv1, PREFIX[1], 3, 1001)
    for i, t in enumerate(run):
        ref1 = dec.row(t, PREFIX[1] + i, kv1)
    kv3 = dec.new_kv()
    prefix_kv(ops, oracle, dec, kv3, PREFIX[3], 3, 1003)
    ref3 = dec.row(42, PREFIX[3], kv3)
    for compact, ref in ((0, ref1), (1, ref3)):
        assert np.array_equal(small.batch_logits_row(compact), ref), f"compact row {compact}"
    assert small.slot_length(1) == PREFIX[1] + 5


def test_batch_invariance(small):
    """BatchedDecodeTests: a row's logits are bit-identical alone, in a batch,
    and with the batch reordered (BatchedDecodeTests.cs:40-45,61-132)."""
    _fresh(small)
    small.forward_batch([77], [2], [0])
    alone = small.batch_logits_row(0)
    _fresh(small)
    small.forward_batch([5, 77, 9], [0, 2, 3], [0, 1, 2])
    batched = small.batch_logits_row(1)
    _fresh(small)
    small.forward_batch([9, 5, 77], [3, 0, 2], [2, 1, 0])
    reordered = small.batch_logits_row(0)
    assert np.array_equal(alone, batched)
    assert np.array_equal(alone, reordered)


def test_mark_rewind_is_bit_identical(small):
    """RewindTests: rewind to a mark then replay gives identical logits."""
    _fresh(small)
    small.mark_slot(1)
    small.forward_batch([3, 4, 5], [1, 1, 1], [2])
    first = small.batch_logits_row(0)
    small.rewind_slot(1)
    assert small.slot_length(1) == PREFIX[1]
    small.forward_batch([3, 4, 5], [1, 1, 1], [2])
    assert np.array_equal(first, small.batch_logits_row(0))


def test_context_exhausted_and_bad_args(small, pkg):
    from needle_cs_b200 import NeedleError

    _fresh(small)
    small.reset_slot(5)
    small.fill_synthetic(5, 255, 3, 77)
    small.forward_batch([1], [5], [0])  # position 255 is the last one
    with pytest.raises(NeedleError) as e:
        small.forward_batch([1], [5], [0])
    assert e.value.status == 3  # ContextExhausted
    with pytest.raises(NeedleError) as e:
        small.forward_batch([1, 2], [0, 9], [0])
    assert e.value.status == 100
    with pytest.raises(NeedleError) as e:
        small.forward_batch([5000], [0], [0])
    assert e.value.status == 100
    with pytest.raises(NeedleError):
        small.feed_slot(5, [1, 2])


def test_masked_argmax_and_probability(small, oracle):
    _fresh(small)
    small.forward_batch([1, 2, 3, 4], [0, 1, 2, 3], [0, 1, 2, 3])
    rng = np.random.default_rng(5)
    words = (small.vocab_size + 31) // 32
    masks = rng.integers(0, 2 ** 32, (4, words), dtype=np.uint64).astype(np.uint32)
    masks[1] = 0  # nothing allowed -> -1
    masks[2, :] = 0
    masks[2, 3] = 1 << 7  # a single allowed id
    ids, probs = small.sample_argmax(masks, with_probs=True)
    for r in range(4):
        logits = small.batch_logits_row(r)
        best, p = oracle.argmax_masked_with_probability(logits, masks[r], small.vocab_size)
        assert ids[r] == best
        assert abs(probs[r] - p) <= 1e-5 * max(p, 1e-30) + 1e-7
    assert ids[1] == -1 and probs[1] == 0.0
    assert ids[2] == 3 * 32 + 7 and probs[2] == 1.0


def test_topk_logsoftmax(small, oracle):
    _fresh(small)
    small.forward_batch([1, 2], [0, 1], [0, 1])
    ids, lp, pr = small.sample_topk(3, mask_special_023=True, with_probs=True)
    for r in range(2):
        ri, rl, rp = oracle.topk_logsoftmax(small.batch_logits_row(r), 3, mask_special_023=True)
        assert list(ids[r]) == list(ri)
        assert np.allclose(lp[r], rl, atol=1e-5)
        assert np.allclose(pr[r], rp, rtol=1e-5)


def test_host_generation_matches_device(small):
    """needle_cs_b200.synthetic rebuilds the engine's device weights bit for bit."""
    import importlib

    syn = importlib.import_module("needle_cs_b200.synthetic")
    layers, fnorm, emb, wh, sh = syn.decoder_weights(small.model)
    for l, t in enumerate(layers):
        for name, arr in t.items():
            got = small.read_tensor(name, arr.dtype, layer=l)
            assert np.array_equal(got, arr), (l, name)
    assert np.array_equal(small.read_tensor("final_norm", np.float32), fnorm)
    assert np.array_equal(small.read_tensor("embedding", np.uint16), emb)
    assert np.array_equal(small.read_tensor("w_head", np.int8), wh)
    assert np.array_equal(small.read_tensor("s_head", np.uint16), sh)


def test_decode_long_sessions_eight_heads(pkg, ops, oracle, cuda):
    """The benchmark geometry (8 heads x 64, d 512) with long ragged sessions
    (up to 1000 positions, 16 pages per (row, head))."""
    import importlib

    eng_mod = importlib.import_module("needle_cs_b200.engine")
    model = eng_mod.SyntheticDecoder(layers=2, dim=512, heads=8, head_dim=64, ffn=512, vocab=2048, seed=21)
    prefix = [300, 1000, 64, 777]
    with eng_mod.BatchedEngine(model, slots=4, context_length=1088, chunk_size=8) as eng:
        for s, n in enumerate(prefix):
            eng.fill_synthetic(s, n, 9, 500 + s)
        tokens = [17, 1999, 3, 1024]
        eng.forward_batch(tokens, [0, 1, 2, 3], [0, 1, 2, 3])
        ids = eng.sample_argmax()
        dec = oracle_decoder(oracle, eng)
        for s, n in enumerate(prefix):
            kv = dec.new_kv()
            prefix_kv(ops, oracle, dec, kv, n, 9, 500 + s)
            ref = dec.row(tokens[s], n, kv)
            assert np.array_equal(eng.batch_logits_row(s), ref), f"slot {s}"
            assert ids[s] == int(np.argmax(ref)), f"slot {s}: margin {top2_margin(ref)}"


def test_graph_replay_matches_direct_launches(small):
    """A step replayed from the captured CUDA graph equals direct launches bit for bit."""
    small.use_graphs(False)
    _fresh(small)
    small.forward_batch([5, 77, 9], [0, 2, 3], [0, 1, 2])
    direct = [small.batch_logits_row(i) for i in range(3)]
    small.use_graphs(True)
    for _ in range(2):  # capture, then replay
        _fresh(small)
        small.forward_batch([5, 77, 9], [0, 2, 3], [0, 1, 2])
        for i in range(3):
            assert np.array_equal(small.batch_logits_row(i), direct[i])


def test_overlapped_launches_match_serial_launches(small):
    """Programmatic dependent launch only overlaps launch latency: logits with
    it on (graphs and direct launches) equal those with it off, bit for bit."""
    small.use_pdl(False)
    small.use_graphs(False)
    _fresh(small)
    small.forward_batch([5, 77, 9, 100], [0, 2, 3, 3], [0, 1, 3])
    serial = [small.batch_logits_row(i) for i in range(3)]
    small.use_pdl(True)
    for graphs in (False, True, True):
        small.use_graphs(graphs)
        _fresh(small)
        small.forward_batch([5, 77, 9, 100], [0, 2, 3, 3], [0, 1, 3])
        for i in range(3):
            assert np.array_equal(small.batch_logits_row(i), serial[i]), (graphs, i)
    small.use_graphs(True)
