"""The decoders bench.py times, against the CPU oracle over many greedy steps.

The 12-layer synthetic decoder (d 512, 8x64 heads, SwiGLU 2048, vocab 8192,
model seed 1) in the two shapes the benchmark measures:
* cfg2: 64 sessions, KV lengths U[16,512] (prefix seed 1), one 64-row batch;
* cfg5: the first 512-row batch of the per-GPU 1024 sessions, KV lengths
  U[64,1024] (prefix seed 5); every 32nd session is replayed on the oracle.
Sessions, lengths and first tokens are drawn exactly as bench.py draws them.
Every step feeds each row's greedy id back, 16 steps in a row.  Bars: the
token ids of every checked session are identical to the oracle's at every
step (ParityTests.cs:80-100 greedy generation) and every logit is
bit-identical to the oracle's (BASELINE's bar is max-abs 1e-3 / rel 1e-2;
each kernel of the step keeps the reference's rounding order, so the
12-layer chain does not drift at all).
"""
import numpy as np
import pytest

from decoder_support import oracle_decoder, oracle_greedy, parallel_map

pytestmark = pytest.mark.gpu

STEPS = 16
PRESETS = {  # bench.py DecodeWorkload.PRESETS
    "cfg2": dict(sessions=64, rows=64, lo=16, hi=512, seed=1, check_every=1),
    "cfg5": dict(sessions=1024, rows=512, lo=64, hi=1024, seed=5, check_every=32),
}


def _layout(p):
    """bench.py DecodeWorkload.global_layout at one rank."""
    lengths = np.random.default_rng(p["seed"]).integers(p["lo"], p["hi"] + 1, size=p["sessions"])
    tokens = np.random.default_rng(p["seed"] + 1).integers(0, 8192, size=p["sessions"]).astype(np.int32)
    return lengths[:p["rows"]], tokens[:p["rows"]]


@pytest.mark.parametrize("preset", ["cfg2", "cfg5"])
def test_benchmark_decoder_greedy_matches_oracle(pkg, ops, oracle, cuda, preset):
    from needle_cs_b200.engine import BatchedEngine, SyntheticDecoder

    p = PRESETS[preset]
    lengths, tokens = _layout(p)
    n = p["rows"]
    checked = list(range(0, n, p["check_every"]))
    cap = ((p["hi"] + STEPS + 63) // 64) * 64
    model = SyntheticDecoder(seed=1)
    assert (model.layers, model.dim, model.vocab) == (12, 512, 8192)
    with BatchedEngine(model, slots=n, context_length=cap, chunk_size=n, max_heads=n) as eng:
        for j in range(n):
            eng.fill_synthetic(j, int(lengths[j]), p["seed"], j)
        slots = np.arange(n, dtype=np.int32)
        toks = tokens.copy()
        gpu_ids = np.zeros((STEPS, n), np.int32)
        gpu_logits = {r: [] for r in checked}
        for s in range(STEPS):
            eng.forward_batch(toks, slots, slots)
            ids = eng.sample_argmax()
            for r in checked:
                gpu_logits[r].append(eng.batch_logits_row(r))
            gpu_ids[s] = ids
            toks = ids.astype(np.int32)
        dec = oracle_decoder(oracle, eng)

    def replay(r):
        return oracle_greedy(ops, oracle, dec, p["seed"], r, int(lengths[r]), int(tokens[r]), STEPS)

    results = parallel_map(replay, checked)
    for r, (ids, logits) in zip(checked, results):
        assert list(gpu_ids[:, r]) == ids, (r, list(gpu_ids[:, r]), ids)
        for s in range(STEPS):
            got, ref = gpu_logits[r][s], logits[s]
            assert np.array_equal(got, ref), (r, s, float(np.abs(got - ref).max()))
