"""Primed prefixes on the GPU: export / import (Engine.ExportPrimedPrefix /
ImportPrimedPrefix, src/Needle/Engine.cs:398-464) and prefix sharing.

Bars: the exported blob equals the reference layout built from the oracle's
own quantization of the same synthetic prefix, byte for byte; an imported or
shared prefix decodes bit-identically to a slot that holds the same prefix on
its own; slots that share pages stay independent; pages return to the pool
when the last slot holding them lets go.
"""
import numpy as np
import pytest

from decoder_support import oracle_decoder, prefix_kv, read_slot_kv

pytestmark = pytest.mark.gpu

SMALL = dict(layers=2, dim=128, heads=2, head_dim=64, ffn=256, vocab=1000, seed=7)
SEED, SESSION = 3, 41


@pytest.fixture(scope="module")
def eng(pkg, cuda):
    import importlib

    eng_mod = importlib.import_module("needle_cs_b200.engine")
    e = eng_mod.BatchedEngine(eng_mod.SyntheticDecoder(**SMALL), slots=8, context_length=512, chunk_size=16)
    yield e
    e.close()


def _reset(eng):
    for s in range(eng.slots):
        eng.reset_slot(s)


def _primed(eng, slot, n, seed=SEED, session=SESSION):
    eng.fill_synthetic(slot, n, seed, session)
    eng.mark_slot(slot)


def reference_blob(kv, layers, n):
    """int32 length, then per layer keys, values, key scales, value scales
    (Engine.ExportPrimedPrefix's order and row layout)."""
    parts = [np.array([n], np.int32).tobytes()]
    for l in range(layers):
        parts += [kv["k"][l, :n].tobytes(), kv["v"][l, :n].tobytes(), kv["ks"][l, :n].tobytes(),
                  kv["vs"][l, :n].tobytes()]
    return b"".join(parts)


def _decode(eng, tokens, slots):
    eng.forward_batch(tokens, slots, list(range(len(slots))))
    return [eng.batch_logits_row(i).copy() for i in range(len(slots))]


@pytest.mark.parametrize("n", [1, 64, 150])
def test_export_matches_reference_layout(eng, ops, oracle, n):
    _reset(eng)
    _primed(eng, 0, n)
    blob = eng.export_prefix(0)
    L, H = SMALL["layers"], SMALL["heads"]
    assert eng.prefix_bytes(0) == len(blob) == 4 + L * n * (2 * H * 64 + 8 * H)
    dec = oracle_decoder(oracle, eng)
    kv = dec.new_kv()
    prefix_kv(ops, oracle, dec, kv, n, SEED, SESSION)
    assert blob == reference_blob(kv, L, n)


def test_export_empty_prefix(eng):
    _reset(eng)
    blob = eng.export_prefix(3)
    assert blob == np.array([0], np.int32).tobytes()


def test_import_round_trip_decodes_identically(eng):
    _reset(eng)
    _primed(eng, 0, 150)
    blob = eng.export_prefix(0)
    eng.import_prefix(1, blob)
    assert eng.slot_length(1) == 150
    a, b = read_slot_kv(eng, 0, 150), read_slot_kv(eng, 1, 150)
    for key in ("k", "v", "ks", "vs"):
        assert np.array_equal(a[key], b[key]), key
    assert eng.export_prefix(1) == blob
    for step in range(3):  # the two slots decode the same tokens bit-identically
        la, lb = _decode(eng, [11 + step, 11 + step], [0, 1])
        assert np.array_equal(la, lb), step


def test_import_rejects_bad_blobs(eng):
    from needle_cs_b200 import NeedleError

    _reset(eng)
    _primed(eng, 0, 70)
    blob = eng.export_prefix(0)
    with pytest.raises(NeedleError) as e:  # truncated
        eng.import_prefix(1, blob[:-1])
    assert e.value.status == 100
    too_long = np.array([eng.capacity + 1], np.int32).tobytes() + blob[4:]
    with pytest.raises(NeedleError) as e:  # longer than the context
        eng.import_prefix(1, too_long)
    assert e.value.status == 100


def test_shared_prefix_decodes_like_an_own_copy(eng):
    _reset(eng)
    free0 = eng.free_pages()
    _primed(eng, 0, 150)  # pages 0, 1 whole, page 2 holds positions 128..149
    eng.share_prefix(1, 0)
    eng.share_prefix(2, 0)
    assert eng.slot_length(1) == eng.slot_length(2) == 150
    assert eng.free_pages() == free0 - 3 - 1 - 1  # the whole pages are held once
    _primed(eng, 3, 150)  # reference slots with their own copies
    _primed(eng, 4, 150)
    _primed(eng, 5, 150)
    for step in range(70):  # past the next page boundary (192)
        t = [5 + step, 600 + step, 900 - step]
        got = _decode(eng, t + t, [0, 1, 2, 3, 4, 5])
        for i in range(3):
            assert np.array_equal(got[i], got[3 + i]), (step, i)


def test_shared_pages_survive_the_source(eng):
    _reset(eng)
    _primed(eng, 0, 130)
    eng.share_prefix(1, 0)
    _primed(eng, 2, 130)
    eng.reset_slot(0)  # the source lets go; slot 1 still holds the shared pages
    _primed(eng, 0, 200, seed=9, session=5)  # reuses freed pages for other content
    for step in range(4):
        got = _decode(eng, [7 + step, 7 + step], [1, 2])
        assert np.array_equal(got[0], got[1]), step


def test_pages_return_to_the_pool(eng):
    _reset(eng)
    free0 = eng.free_pages()
    _primed(eng, 0, 300)
    for s in range(1, 6):
        eng.share_prefix(s, 0)
    _decode(eng, [1, 2, 3, 4, 5, 6], [0, 1, 2, 3, 4, 5])
    assert eng.free_pages() < free0
    _reset(eng)
    assert eng.free_pages() == free0
