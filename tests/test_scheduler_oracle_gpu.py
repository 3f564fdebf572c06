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


def _oracle_with_forced(oracle, dec, prompt, max_new, mask, vocab, force_at, forced):
    """oracle_request with jump-forward: after the request's force_at-th pick
    the forced tokens join the output (no sample) and are fed in order."""
    kv = dec.new_kv()
    pos = 0
    for t in prompt:
        logits = dec.row(int(t), pos, kv)
        pos += 1
    out = []
    while len(out) < max_new:
        tok = int(oracle.argmax_masked(logits, mask, vocab))
        out.append(tok)
        feed = [tok] + (list(forced) if len(out) == force_at else [])
        if len(out) == force_at:
            out += list(forced)
        if len(out) >= max_new:
            break
        for t in feed:
            logits = dec.row(int(t), pos, kv)
            pos += 1
    return out[:max_new]


def test_jump_forward_streams_equal_oracle(pkg, oracle, cuda):
    """Grammar-forced tokens fed as one run (ndl_sched_force; NeedleSession's
    jump-forward, src/Needle/NeedleSession.cs:538-662) give every request the
    stream of its oracle replay with the same tokens forced, and the same
    stream as without the jump: a run equals feeding its tokens one per step."""
    from needle_cs_b200.engine import BatchedEngine, SyntheticDecoder
    from needle_cs_b200.scheduler import Scheduler

    rng = np.random.default_rng(41)
    model = SyntheticDecoder(layers=2, seed=1)
    V = model.vocab
    words = (V + 31) // 32
    reqs = {}
    for rid in range(3):
        bits = rng.random(V) < 0.3
        mask = np.zeros(words, np.uint32)
        for i in np.nonzero(bits)[0]:
            mask[i >> 5] |= np.uint32(1 << (i & 31))
        forced = [int(t) for t in rng.integers(0, V, 3 + rid)]
        reqs[rid] = (rng.integers(0, V, int(rng.integers(8, 40))).astype(np.int32), 14, mask, 3 + rid, forced)
    with BatchedEngine(model, slots=4, context_length=128, chunk_size=64, max_heads=64) as eng:
        sched = Scheduler(eng, max_rows=64, prefill_chunk=64)
        for rid, (p, mn, m, _, _) in reqs.items():
            sched.submit(rid, p, mn, mask=m)
        forced_done = set()
        for _ in range(100):
            w, r = sched.pending()
            if w == 0 and r == 0:
                break
            sched.step()
            for rid, (_, _, _, at, forced) in reqs.items():
                if rid not in forced_done and len(sched.tokens(rid)) == at:
                    sched.force(rid, forced)
                    forced_done.add(rid)
        assert forced_done == set(reqs)
        streams = {rid: [int(t) for t in sched.tokens(rid)] for rid in reqs}
        sched.close()
        dec = oracle_decoder(oracle, eng)
    for rid, (p, mn, m, at, forced) in reqs.items():
        want = _oracle_with_forced(oracle, dec, p, mn, m, V, at, forced)
        assert streams[rid] == want, (rid, streams[rid], want)
        assert streams[rid][at:at + len(forced)] == forced
