"""Continuous batching on the benchmarked decoder against the CPU oracle.

The 12-layer synthetic decoder of cfg3 serves 8 requests through the
scheduler (ndl_sched_*): prompts U[32,384] tokens (longer ones split into
256-row prefill chunks), arrivals spread over the first steps so prefill
chunks and decode rows share steps, every request with its own vocabulary
bitmask (30 % of the ids allowed).  Each request's token stream must equal
the oracle's replay of that request alone (the reference's contract:
BatchedSession results equal sequential sessions,
tests/Needle.Tests/BatchedDecodeTests.cs:172-258).
"""
import numpy as np
import pytest

from decoder_support import oracle_decoder, oracle_request, parallel_map

pytestmark = pytest.mark.gpu


def test_scheduler_streams_equal_oracle_replays(pkg, oracle, cuda):
    from needle_cs_b200.engine import BatchedEngine, SyntheticDecoder
    from needle_cs_b200.scheduler import FINISHED, Scheduler

    rng = np.random.default_rng(33)
    model = SyntheticDecoder(seed=1)
    V = model.vocab
    words = (V + 31) // 32
    reqs = {}
    for rid in range(8):
        prompt = rng.integers(0, V, int(rng.integers(32, 385))).astype(np.int32)
        bits = rng.random(V) < 0.3
        mask = np.zeros(words, np.uint32)
        for i in np.nonzero(bits)[0]:
            mask[i >> 5] |= np.uint32(1 << (i & 31))
        reqs[rid] = (prompt, int(rng.integers(8, 25)), mask)
    assert any(len(p) > 256 for p, _, _ in reqs.values())  # at least one prompt is split into chunks
    with BatchedEngine(model, slots=8, context_length=448, chunk_size=512, max_heads=512) as eng:
        sched = Scheduler(eng, max_rows=512, prefill_chunk=256)
        order = list(reqs)
        submitted, steps, done, mixed = 0, 0, {}, 0
        while True:
            while submitted < len(order) and submitted <= 2 * steps:
                rid = order[submitted]
                p, mn, m = reqs[rid]
                sched.submit(rid, p, mn, mask=m)
                submitted += 1
            w, r = sched.pending()
            if submitted == len(order) and w == 0 and r == 0:
                break
            ev, rows, dec_rows = sched.step()
            mixed += int(0 < dec_rows < rows)
            steps += 1
            for rid, kind, tok, st in ev:
                if kind == FINISHED:
                    done[rid] = st
            assert steps < 1000
        streams = {rid: [int(t) for t in sched.tokens(rid)] for rid in reqs}
        sched.close()
        dec = oracle_decoder(oracle, eng)
    assert sorted(done) == sorted(reqs) and all(v == 0 for v in done.values())
    assert mixed > 0  # some steps packed prefill chunks beside decode rows
    replays = parallel_map(lambda rid: oracle_request(oracle, dec, reqs[rid][0], reqs[rid][1], reqs[rid][2], V),
                           order)
    for rid, ref in zip(order, replays):
        assert streams[rid] == ref, (rid, streams[rid], ref)
        m = reqs[rid][2]
        assert all((int(m[t >> 5]) >> (t & 31)) & 1 for t in ref)
