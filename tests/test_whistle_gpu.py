"""The Whistle encoder on the GPU (ndl_whistle_*: Whistle.Encode and
BuildCrossMemory, src/Needle/Whistle.cs:179-200, 886-914) against the CPU
oracle's scalar chain (oracle/whistle.py) on a synthetic archive with an
audio section and seeded synthetic audio.

Bar: bit-identical at every stage (the normalized log-mel features, the stem
rows, the encoder output, every decoder layer's int8 cross keys / values and
their scales): both sides take the scalar tier's operations one rounding at a
time, MathF.Exp and MathF.Log correctly rounded.
"""
import numpy as np
import pytest

from cact_support import whistle_archive
from whistle_support import speech_like, whistle_oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def whistle(pkg):
    import importlib

    cact = importlib.import_module("needle_cs_b200.model")
    wmod = importlib.import_module("needle_cs_b200.whistle")
    a = whistle_archive(seed=3)
    m = cact.Model(a.build(), device=0)
    w = wmod.Whistle(m, max_seconds=4)
    yield a, m, w
    w.close()
    m.close()


def _bits(x):
    return np.ascontiguousarray(x).view(np.uint32)


@pytest.mark.parametrize("seconds,seed", [(1.0, 0), (2.37, 1), (0.012, 2)])
def test_encoder_matches_the_scalar_chain(whistle, seconds, seed):
    a, _, w = whistle
    pcm = speech_like(seconds, seed=seed)
    o = whistle_oracle(a)
    want = o.encode(pcm)
    got = w.encode(pcm)
    assert got == want
    assert np.array_equal(_bits(w.mel()), _bits(o.mel))
    if want == 0:
        return
    assert np.array_equal(_bits(w.stem()), _bits(o.stem_out))
    enc = w.encoder_output()
    assert np.isfinite(enc).all() and np.abs(enc).max() > 0.1
    assert np.array_equal(_bits(enc), _bits(o.encoder_out))
    for layer, (keys, ks, vals, vs) in enumerate(o.build_memory()):
        gk, gks, gv, gvs = w.memory(layer)
        assert np.array_equal(gk, keys) and np.array_equal(gv, vals), layer
        assert np.array_equal(_bits(gks), _bits(ks)) and np.array_equal(_bits(gvs), _bits(vs)), layer


def test_under_one_hop_and_limits(whistle):
    from needle_cs_b200 import NeedleError

    _, m, w = whistle
    assert w.encode(np.zeros(100, np.float32)) == 0  # fewer samples than one hop: no frames
    with pytest.raises(NeedleError):
        import ctypes

        from needle_cs_b200._native import call
        call("ndl_whistle_encode_device", w._h, None, 10 ** 8)  # beyond max_samples
