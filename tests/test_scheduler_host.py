"""Step packing of the continuous-batching scheduler, on the host (a dry
scheduler: no engine, deterministic fake sampling).

Invariants of BatchedSession.RunBatch (src/Needle/BatchedSession.cs:218-268)
kept by the mixed scheduler: every running request's rows are contiguous and
in position order, a step never exceeds its row budget, decode rows come
first, prompts are fed in chunks of at most prefill_chunk positions, the
prompt's last position is the head row that yields the first token, and a
request whose slot would pass the capacity ends with ContextExhausted (3).
"""
import numpy as np
import pytest

from conftest import entry


@pytest.fixture(scope="module")
def sched_mod(pkg):
    import importlib
    return importlib.import_module("needle_cs_b200.scheduler")


def _run(sched, max_steps=10000):
    plans, events = [], []
    for _ in range(max_steps):
        w, r = sched.pending()
        if w == 0 and r == 0:
            break
        ev, rows, dec = sched.step()
        plans.append((sched.last_plan(), rows, dec))
        events.extend(ev)
    return plans, events


def test_packing_invariants(sched_mod):
    rng = np.random.default_rng(7)
    vocab, slots, cap = 1000, 6, 512
    s = sched_mod.Scheduler(None, max_rows=64, prefill_chunk=40, slots=slots, capacity=cap, vocab=vocab)
    prompts, max_new = {}, {}
    for rid in range(15):
        n = int(rng.integers(1, 150))
        prompts[rid] = rng.integers(0, vocab, n).astype(np.int32)
        max_new[rid] = int(rng.integers(1, 12))
        s.submit(rid, prompts[rid], max_new[rid])
    plans, events = _run(s)
    fed = {rid: 0 for rid in prompts}
    for (tokens, row_slots, heads), rows, dec in plans:
        assert rows == len(tokens) <= 64
        # contiguous runs per slot
        seen, prev = set(), None
        for sl in row_slots:
            if sl != prev:
                assert sl not in seen
                seen.add(sl)
                prev = sl
        # decode rows lead the step and are all head rows
        assert list(heads[:dec]) == list(range(dec))
        runs = {}
        for i, sl in enumerate(row_slots):
            runs.setdefault(int(sl), []).append(i)
        for sl, idx in runs.items():
            if idx[0] < dec:
                assert len(idx) == 1
            else:
                assert len(idx) <= 40
    firsts = [e for e in events if e[1] == 1]
    dones = [e for e in events if e[1] == 2]
    assert sorted(e[0] for e in firsts) == sorted(prompts)
    assert sorted(e[0] for e in dones) == sorted(prompts)
    for rid in prompts:
        toks = s.tokens(rid)
        assert len(toks) == max_new[rid]
        assert list(toks) == [(rid * 7919 + i) % vocab for i in range(max_new[rid])]
        fi = [i for i, e in enumerate(events) if e[0] == rid and e[1] == 1][0]
        di = [i for i, e in enumerate(events) if e[0] == rid and e[1] == 2][0]
        assert fi <= di and events[di][3] == 0


def test_prompt_chunks_and_first_token(sched_mod):
    s = sched_mod.Scheduler(None, max_rows=16, prefill_chunk=8, slots=2, capacity=256, vocab=50)
    s.submit(3, np.arange(20) % 50, 2)
    rows_seen = []
    while True:
        ev, rows, dec = s.step()
        t, sl, h = s.last_plan()
        rows_seen.append((rows, list(h)))
        if any(e[1] == 2 for e in ev):
            break
    # 20 prompt positions in chunks of 8, 8, 4; the last chunk's last row is the head row
    assert rows_seen[:3] == [(8, []), (8, []), (4, [3])]
    assert rows_seen[3] == (1, [0])
    assert list(s.tokens(3)) == [(3 * 7919) % 50, (3 * 7919 + 1) % 50]


def test_context_exhausted_and_slot_reuse(sched_mod):
    s = sched_mod.Scheduler(None, max_rows=32, prefill_chunk=32, slots=1, capacity=20, vocab=100)
    s.submit(0, np.zeros(18, np.int32), 10)   # 18 prompt + 10 new > 20
    s.submit(1, np.zeros(4, np.int32), 2)     # waits for the only slot
    plans, events = _run(s)
    done = {e[0]: e for e in events if e[1] == 2}
    assert done[0][3] == 3                    # ContextExhausted
    assert len(s.tokens(0)) == 20 - 18 + 1    # positions 18, 19 decoded, then the 21st would not fit
    assert done[1][3] == 0 and len(s.tokens(1)) == 2


def test_rejects_bad_requests(sched_mod):
    from needle_cs_b200 import NeedleError

    s = sched_mod.Scheduler(None, max_rows=8, prefill_chunk=8, slots=1, capacity=64, vocab=10)
    with pytest.raises(NeedleError):
        s.submit(0, [11], 1)                  # token outside the vocabulary
    s.submit(0, [1], 1)
    with pytest.raises(NeedleError):
        s.submit(0, [1], 1)                   # duplicate id


def test_jump_forward_runs(sched_mod):
    """Forced tokens (NeedleSession.GenerateCalls' jump-forward,
    src/Needle/NeedleSession.cs:538-662) join the request's output without a
    sample; the next step feeds the last pick and the forced tokens as one
    contiguous run of the request's slot with the head at its last row; they
    count toward max_new_tokens, and a stop token among them ends the request."""
    from needle_cs_b200._native import NeedleError

    vocab = 1000
    s = sched_mod.Scheduler(None, max_rows=8, prefill_chunk=8, slots=2, capacity=64, vocab=vocab)
    s.submit(0, np.arange(3, dtype=np.int32), 12)
    s.submit(1, np.arange(5, dtype=np.int32), 6, stop_token=77)
    with pytest.raises(NeedleError):  # not decoding yet
        s.force(0, [5])
    s.step()  # both prompts, first tokens
    s.step()  # one decode row each
    out0 = list(s.tokens(0))
    assert len(out0) == 2
    s.force(0, [501, 502, 503])
    ev, rows, dec = s.step()
    tokens, row_slots, heads = s.last_plan()
    r0 = [i for i, sl in enumerate(row_slots) if sl == row_slots[0]]
    assert [int(tokens[i]) for i in r0] == [out0[-1], 501, 502, 503]  # the pick, then the forced run
    assert r0 == list(range(r0[0], r0[0] + 4)) and r0[-1] in list(heads)
    assert list(s.tokens(0))[:5] == out0 + [501, 502, 503]
    assert len(s.tokens(0)) == 6  # and the run's sample
    # a run longer than the step's free rows is split; the head waits for its last row
    s.force(0, list(range(600, 612))[:5])
    ev, rows, dec = s.step()
    assert rows <= 8
    # the stop token among forced tokens ends request 1 at the next step
    s.force(1, [5, 77])
    ev, rows, dec = s.step()
    finished = [e for e in ev if e[0] == 1 and e[1] == sched_mod.FINISHED]
    assert finished and finished[0][2] == 77
    assert list(s.tokens(1))[-2:] == [5, 77]
    with pytest.raises(NeedleError):
        s.force(1, [5])  # done
    with pytest.raises(NeedleError):
        s.force(0, [vocab])  # outside the vocabulary
