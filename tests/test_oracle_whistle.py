"""Pins the Whistle encoder's CPU restatement (oracle/whistle.py,
oracle/whistle_oracle.c) against independent formulations: numpy's float64
FFT for the mel front end, float64 logarithms, the column statistics of
Normalize, a float64 convolution for the first stem stage, and the archive
writer's record kinds for the AudioWeights walk.  The reference's own stage
goldens (tools/golden_whistle.py on whistle.cact) are absent here."""
import ctypes

import numpy as np
import pytest

from cact_support import CQ, whistle_archive
from whistle_support import speech_like, whistle_oracle


@pytest.fixture(scope="module")
def wo(oracle):
    a = whistle_archive(seed=7)
    return a, whistle_oracle(a)


def test_log_rn_is_the_rounded_double_log(oracle):
    lib = oracle.lib()
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.uniform(1e-38, 1e-30, 2000), rng.uniform(1e-3, 10, 20000),
                        np.exp(rng.uniform(-87, 88, 20000)), [1.0, 2.0, 0.5, 1e-45, 3.4e38]]).astype(np.float32)
    y = np.empty_like(x)
    lib.ndo_log_rn_array(x.ctypes.data, x.size, y.ctypes.data)
    assert np.array_equal(y, np.log(x.astype(np.float64)).astype(np.float32))
    assert np.isneginf(lib.ndo_log_rn(0.0)) and np.isnan(lib.ndo_log_rn(-1.0))


def test_mel_frames_match_float64_fft(wo, oracle):
    _, o = wo
    lib = oracle.lib()
    fft, window, mels = o.fft, o.window, o.mels
    bank = o.A("mel")
    hann, cs, sn = np.zeros(window, np.float32), np.zeros(fft // 2, np.float32), np.zeros(fft // 2, np.float32)
    bitrev, first, count = (np.zeros(fft, np.int32), np.zeros(fft // 2 + 1, np.int32),
                            np.zeros(fft // 2 + 1, np.int32))
    lib.ndo_frontend_tables(fft, window, bank.ctypes.data, mels, hann.ctypes.data, cs.ctypes.data, sn.ctypes.data,
                            bitrev.ctypes.data, first.ctypes.data, count.ctypes.data)
    assert np.array_equal(np.sort(bitrev), np.arange(fft))
    seg = np.zeros(fft, np.float32)
    seg[:window] = speech_like(0.05, seed=3)[:window]
    got = np.zeros(mels, np.float32)
    peak = lib.ndo_mel_frame(seg.ctypes.data, fft, window, hann.ctypes.data, cs.ctypes.data, sn.ctypes.data,
                             bitrev.ctypes.data, bank.ctypes.data, mels, first.ctypes.data, count.ctypes.data,
                             got.ctypes.data)
    w64 = 0.5 - 0.5 * np.cos(2 * np.pi * np.arange(window) / (window - 1))
    spec = np.fft.rfft(np.concatenate([seg[:window] * w64, np.zeros(fft - window)]))
    want = (np.abs(spec) ** 2) @ bank.reshape(fft // 2 + 1, mels).astype(np.float64)
    assert np.allclose(got, want, rtol=1e-4, atol=1e-6 * want.max())
    assert peak == got.max()


def test_features_are_normalized_log_mels(wo):
    _, o = wo
    l0, feats = o.features(speech_like(1.3, seed=4))
    assert l0 == int(1.3 * 16000) // o.hop and feats.shape == (l0, o.mels)
    assert np.abs(feats.mean(0)).max() < 1e-5
    assert np.abs(feats.std(0, ddof=1) - 1).max() < 1e-4


def test_first_stem_stage_matches_float64_conv(wo):
    _, o = wo
    _, feats = o.features(speech_like(0.6, seed=5))
    s, mels, l0 = o.stem_width, o.mels, feats.shape[0]
    w = o.A("stem_first").reshape(3, 3, s).astype(np.float64)
    padded = np.zeros((l0 + 2, mels + 2))
    padded[1:-1, 1:-1] = feats
    l1 = (l0 + 1) // 2
    conv = np.zeros((l1, 40, s))
    for dt in range(3):
        for df in range(3):
            rows = padded[2 * np.arange(l1) + dt][:, 2 * np.arange(40) + df]  # rows 2p - 1 + dt, bins 2f - 1 + df
            conv += rows[:, :, None] * w[dt, df][None, None, :]
    want = conv * (1 / (1 + np.exp(-conv)))
    # the oracle's stage 1 (AddScaled in float32, SiLU with a correctly rounded exp)
    got = np.zeros((l1, 40, s), np.float32)
    first = o.A("stem_first").reshape(9, s)
    for p in range(l1):
        out = np.zeros((40, s), np.float32)
        for dt in range(3):
            r = 2 * p - 1 + dt
            row = feats[r] if 0 <= r < l0 else np.zeros(mels, np.float32)
            for df in range(3):
                freq = 2 * np.arange(40) - 1 + df
                ok = (freq >= 0) & (freq < mels)
                out[ok] = out[ok] + row[freq[ok]][:, None] * first[dt * 3 + df][None, :]
        got[p] = out
    import oracle.oracle as O
    O.lib().ndo_silu(got.ctypes.data, got.size)
    assert np.allclose(got, want, rtol=1e-4, atol=1e-4)


def test_audio_walk_matches_the_records(wo):
    a, o = wo
    audio = [r for r in a.records if r[0] == "audio"]
    assert len(audio) == len(o.at)
    for name, k in o.at.items():
        rec = next(r for r in audio if r[1] == k)
        is_cq = rec[2] == CQ
        leaf = name.split(".")[-1]
        assert is_cq == (leaf in ("q", "k", "v", "gate", "out", "pw1", "pw2", "phi_pre", "phi_post", "phi_res",
                                  "stem_pointwise1", "stem_pointwise2", "stem_out")), name


def test_encoder_and_memory_shapes(wo):
    _, o = wo
    frames = o.encode(speech_like(0.9, seed=6))
    l0 = int(0.9 * 16000) // o.hop
    assert frames == (((l0 + 1) // 2 + 1) // 2 + 1) // 2
    assert o.encoder_out.shape == (frames, o.dim) and np.isfinite(o.encoder_out).all()
    mem = o.build_memory()
    g = o.g
    assert len(mem) == g["layers"]
    keys, ks, vals, vs = mem[-1]
    assert keys.shape == (frames, g["heads"] * g["qk_dim"]) and vals.shape == (frames, g["heads"] * g["v_dim"])
    assert (ks > 0).all() and (vs > 0).all() and np.abs(keys).max() == 127
    assert o.encode(np.zeros(100, np.float32)) == 0
