"""Whistle-shaped decoder (cfg4): cross memory, cross-attention decode and
beam search against the CPU oracle.

* memory K/V pages: bit-exact int8 and scales vs the oracle's
  BuildCrossMemory restatement (per-frame QuantizeInt8 -> I8G32 W_ckv ->
  per-(frame, head) QuantizeInt8) on the same fp16 memory;
* decode logits with cross-attention: bit-identical to the oracle's;
* slot copy (the beam fork): the copy continues with identical logits;
* beam search: token sequences identical to the oracle's
  Whistle.BeamSearch restatement, scores within 1e-4.
"""
import numpy as np
import pytest

from decoder_support import oracle_decoder, read_slot_kv

pytestmark = pytest.mark.gpu

PROMPT = [50258, 50259, 50359, 50363]  # a start-of-transcript style prefix


@pytest.fixture(scope="module")
def whistle(pkg, cuda):
    from needle_cs_b200.engine import BatchedEngine, whistle_decoder

    eng = BatchedEngine(whistle_decoder(seed=3), slots=16, context_length=192, chunk_size=16, max_heads=16)
    yield eng
    eng.close()


def _memory(engine, slot, frames, utterance):
    engine.reset_slot(slot)
    engine.fill_memory_synthetic(slot, frames, engine.model.seed, utterance)


def _oracle_memory(oracle, dec, engine, frames, utterance):
    from needle_cs_b200.synthetic import memory_values

    mem = memory_values(engine.model.seed, utterance, frames, engine.model.dim)
    return dec.cross_memory(mem)


def test_cross_memory_pages_bit_exact(whistle, oracle):
    dec = oracle_decoder(oracle, whistle)
    for frames, utt in ((130, 5), (64, 6)):
        _memory(whistle, 0, frames, utt)
        got = read_slot_kv(whistle, 0, frames)
        ref = _oracle_memory(oracle, dec, whistle, frames, utt)
        for key in ("k", "v", "ks", "vs"):
            assert np.array_equal(got[key], ref[key]), key


def test_cross_decode_logits_match_oracle(whistle, oracle):
    dec = oracle_decoder(oracle, whistle)
    frames = 100
    _memory(whistle, 0, frames, 9)
    mem = _oracle_memory(oracle, dec, whistle, frames, 9)
    whistle.reset_slot(1)
    whistle.attach_memory(1, 0)
    kv = dec.new_kv()
    toks = PROMPT + [440, 1012, 7, 30000]
    for pos, t in enumerate(toks):
        whistle.forward_batch([t], [1], [0])
        got = whistle.batch_logits_row(0)
        ref = dec.row(t, pos, kv, mem)
        assert np.array_equal(got, ref), (pos, np.abs(got - ref).max())
    # the slot copy continues with the same logits
    whistle.copy_slot(2, 1)
    whistle.forward_batch([77, 77], [1, 2], [0, 1])
    assert np.array_equal(whistle.batch_logits_row(0), whistle.batch_logits_row(1))


def test_beam_search_matches_oracle(whistle, oracle):
    from needle_cs_b200.beam import beam_search

    dec = oracle_decoder(oracle, whistle)
    width, steps = 3, 6
    utts = [(0, 110, 21), (1, 70, 22)]
    mems = []
    for slot, frames, utt in utts:
        _memory(whistle, slot, frames, utt)
        mems.append(_oracle_memory(oracle, dec, whistle, frames, utt))
    beam_slots = np.arange(2, 2 + 2 * width * len(utts)).reshape(len(utts), 2 * width)
    got, scores = beam_search(whistle, [u[0] for u in utts], beam_slots, PROMPT, width=width, max_steps=steps)
    for i, mem in enumerate(mems):
        ref, ref_score = oracle.beam_search(dec, mem, PROMPT, width, steps, eos=50257)
        assert got[i] == ref, (i, got[i], ref)
        assert abs(float(scores[i]) - ref_score) <= 1e-4 * max(1.0, abs(ref_score))


def test_beam_search_full_cfg4_matches_oracle(pkg, oracle, cuda):
    """cfg4's full shape: 1500-frame memories, width 3, up to 128 tokens, on
    4 utterances at once; every utterance's token sequence equals the
    oracle's Whistle.BeamSearch restatement and its score is within 1e-4."""
    from needle_cs_b200.beam import beam_search
    from needle_cs_b200.engine import BatchedEngine, whistle_decoder

    from decoder_support import parallel_map

    width, steps, frames = 3, 128, 1500
    utts = [(u, frames, 40 + u) for u in range(4)]
    with BatchedEngine(whistle_decoder(seed=3), slots=4 + 4 * 2 * width, context_length=1536, chunk_size=16,
                       max_heads=16) as eng:
        for slot, n, utt in utts:
            _memory(eng, slot, n, utt)
        beam_slots = np.arange(4, 4 + 4 * 2 * width).reshape(4, 2 * width)
        got, scores = beam_search(eng, [u[0] for u in utts], beam_slots, PROMPT, width=width, max_steps=steps)
        dec = oracle_decoder(oracle, eng)
        mems = [_oracle_memory(oracle, dec, eng, n, utt) for _, n, utt in utts]

    refs = parallel_map(lambda i: oracle.beam_search(dec, mems[i], PROMPT, width, steps, eos=50257), range(4))
    for i, (ref, ref_score) in enumerate(refs):
        assert got[i] == ref, (i, len(got[i]), len(ref))
        assert abs(float(scores[i]) - ref_score) <= 1e-4 * max(1.0, abs(ref_score))
