"""Continuous batching over one engine (ndl_sched_*).

The step loop of the reference's BatchedSession.RunBatch
(src/Needle/BatchedSession.cs:218-268: collect each lane's pending rows,
one ForwardBatch, advance the lanes, fail a lane with ContextExhausted when
its slot would pass the capacity) with requests admitted as they arrive and
prompt chunks packed beside decode rows.  Greedy masked sampling per request
(Ops.ArgMaxMasked, src/Needle/Ops.cs:1223-1299).
"""
import ctypes

import numpy as np

from ._native import SchedConfig, SchedEvent, call, lib

FIRST_TOKEN, FINISHED = 1, 2


class Scheduler:
    """`engine`: a BatchedEngine, or None for a dry scheduler (no GPU; tokens
    (request * 7919 + produced) % vocab) that only plans steps."""

    def __init__(self, engine=None, max_rows=512, prefill_chunk=256, slots=None, capacity=None, vocab=None):
        cfg = SchedConfig(max_rows, prefill_chunk)
        h = ctypes.c_void_p()
        if engine is not None:
            call("ndl_sched_create", engine.handle, ctypes.byref(cfg), ctypes.byref(h))
            vocab = engine.vocab_size
        else:
            call("ndl_sched_create_dry", ctypes.byref(cfg), slots, capacity, vocab, ctypes.byref(h))
        self._h = h
        self.engine = engine
        self.max_rows = max_rows
        self.vocab = vocab
        self._events = (SchedEvent * 4096)()

    def close(self):
        if self._h:
            lib().ndl_sched_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def submit(self, request, prompt, max_new_tokens, stop_token=-1, mask=None):
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        if mask is None:
            call("ndl_sched_submit", self._h, request, p.ctypes.data, p.size, max_new_tokens, stop_token, None, 0)
        else:
            m = np.ascontiguousarray(mask, dtype=np.uint32)
            call("ndl_sched_submit", self._h, request, p.ctypes.data, p.size, max_new_tokens, stop_token,
                 m.ctypes.data, m.size)

    def force(self, request, tokens):
        """Jump-forward: grammar-forced tokens after the request's last pick
        (ndl_sched_force); the next step feeds them as one run."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        call("ndl_sched_force", self._h, request, t.ctypes.data, t.size)

    def step(self):
        """One step: (events [(request, kind, token, status)], rows, decode_rows)."""
        n, rows, dec = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        call("ndl_sched_step", self._h, self._events, len(self._events), ctypes.byref(n), ctypes.byref(rows),
             ctypes.byref(dec))
        assert n.value <= len(self._events)
        ev = [(e.request, e.kind, e.token, e.status) for e in self._events[:n.value]]
        return ev, rows.value, dec.value

    def tokens(self, request):
        n = ctypes.c_int()
        call("ndl_sched_tokens", self._h, request, None, 0, ctypes.byref(n))
        out = np.empty(n.value, np.int32)
        call("ndl_sched_tokens", self._h, request, out.ctypes.data, n.value, ctypes.byref(n))
        return out

    def pending(self):
        w, r = ctypes.c_int(), ctypes.c_int()
        call("ndl_sched_pending", self._h, ctypes.byref(w), ctypes.byref(r))
        return w.value, r.value

    def last_plan(self):
        t = np.empty(self.max_rows, np.int32)
        s = np.empty(self.max_rows, np.int32)
        hr = np.empty(self.max_rows, np.int32)
        rows, heads = ctypes.c_int(), ctypes.c_int()
        call("ndl_sched_last_plan", self._h, t.ctypes.data, s.ctypes.data, ctypes.byref(rows), hr.ctypes.data,
             ctypes.byref(heads))
        return t[:rows.value], s[:rows.value], hr[:heads.value]
