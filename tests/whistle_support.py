"""The CPU oracle of the Whistle encoder over an archive written by
cact_support.whistle_archive, built from the archive writer's records alone
(dense fp16 audio tensors by Scalar.HalfToSingle, as the loader converts an
audio section; the geometry as the loader derives it)."""
import numpy as np


def whistle_oracle(archive):
    from cact_support import half_to_single
    from oracle.whistle import WhistleOracle

    g = archive.g
    rec = {(r[0], r[1]): r[6] for r in archive.records}
    rows = 1 << ((g["hada_n"] - 1).bit_length() // 2)
    info = dict(g, hada_rows=rows, hada_cols=g["hada_n"] // rows)

    def cq(role, index):
        _, codes, norms, nrows, cols, bits = rec[(role, index)]
        return codes.reshape(nrows, -1), norms.reshape(nrows, -1), nrows, cols, bits

    def dense(role, index=0):
        kind, v = rec[(role, index)][:2]
        return half_to_single(v, exact=True) if kind == "dense16" else np.ascontiguousarray(v, np.float32)

    def perm(role):
        return np.ascontiguousarray(rec[(role, 0)][1], np.int32)

    return WhistleOracle(info, archive.levels, dense, cq, perm)


def speech_like(seconds, rate=16000, seed=0):
    """Seeded synthetic audio: a few gliding harmonics under noise, amplitude
    around 0.1 (the reference's PCM range is [-1, 1])."""
    rng = np.random.default_rng(seed)
    t = np.arange(int(seconds * rate)) / rate
    f0 = 140.0 + 40.0 * np.sin(2 * np.pi * 0.7 * t)
    phase = 2 * np.pi * np.cumsum(f0) / rate
    x = sum(np.sin(k * phase) / k for k in range(1, 6)) * 0.05
    x = x * (0.6 + 0.4 * np.sin(2 * np.pi * 2.3 * t))
    return (x + rng.normal(0, 0.01, t.size)).astype(np.float32)
