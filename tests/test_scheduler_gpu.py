"""Continuous batching on the GPU: mixed prompt chunks and decode rows give
every request exactly the token stream it gets alone.

Each request is replayed on its own through the engine (its prompt fed in
chunks of the engine's row limit, then greedy masked decoding one row at a time, masks passed per
call) and the token ids must be equal; rows are batch invariant, so chunk
boundaries and neighbours must not change a single logit.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _alone(engine, slot, prompt, max_new, mask, stop=-1):
    engine.reset_slot(slot)
    engine.feed_slot(slot, prompt)  # chunks of the engine's row limit
    out = []
    while True:
        tok = int(engine.sample_argmax(mask[None, :] if mask is not None else None)[0])
        if tok < 0:
            break
        out.append(tok)
        if len(out) >= max_new or tok == stop:
            break
        engine.forward_batch([tok], [slot], [0])
    return out


def test_scheduler_streams_equal_single_request_runs(pkg, cuda):
    from needle_cs_b200.engine import BatchedEngine, SyntheticDecoder
    from needle_cs_b200.scheduler import FINISHED, FIRST_TOKEN, Scheduler

    rng = np.random.default_rng(11)
    model = SyntheticDecoder(layers=2, seed=3)
    V = model.vocab
    words = (V + 31) // 32
    eng = BatchedEngine(model, slots=6, context_length=512, chunk_size=96, max_heads=96)
    sched = Scheduler(eng, max_rows=96, prefill_chunk=40)
    reqs = {}
    for rid in range(10):
        n = int(rng.integers(3, 260))
        prompt = rng.integers(0, V, n).astype(np.int32)
        bits = rng.random(V) < 0.3
        mask = np.zeros(words, np.uint32)
        for i in np.nonzero(bits)[0]:
            mask[i >> 5] |= np.uint32(1 << (i & 31))
        reqs[rid] = (prompt, int(rng.integers(2, 14)), mask if rid % 3 else None)
    # arrivals spread over the first steps
    order = list(reqs)
    submitted, steps, firsts, dones = 0, 0, {}, {}
    while True:
        while submitted < len(order) and submitted <= 2 * steps:
            rid = order[submitted]
            p, mn, m = reqs[rid]
            sched.submit(rid, p, mn, mask=m)
            submitted += 1
        w, r = sched.pending()
        if submitted == len(order) and w == 0 and r == 0:
            break
        ev, rows, dec = sched.step()
        steps += 1
        for rid, kind, tok, st in ev:
            if kind == FIRST_TOKEN:
                firsts[rid] = tok
            if kind == FINISHED:
                dones[rid] = st
        assert steps < 2000
    assert sorted(dones) == sorted(reqs) and all(v == 0 for v in dones.values())
    streams = {rid: [int(t) for t in sched.tokens(rid)] for rid in reqs}
    sched.close()
    for rid, (p, mn, m) in reqs.items():
        assert streams[rid][0] == firsts[rid]
        alone = _alone(eng, 0, p, mn, m)
        assert streams[rid] == alone, rid
        if m is not None:
            assert all((int(m[t >> 5]) >> (t & 31)) & 1 for t in streams[rid])
    eng.close()
