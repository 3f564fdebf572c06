"""Beam search of Whistle-shaped decoders over many utterances (ndl_beam_search).

Whistle.BeamSearch (src/Needle/Whistle.Decode.cs:224-350): width beams per
utterance, top-width TopKLogSoftmax expansions (ids 0, 2, 3 masked), EOS ends
a hypothesis, length-normalised scores score/len^penalty; every live beam of
every utterance runs in one batched step.
"""
import ctypes

import numpy as np

from ._native import BeamConfig, call

WHISPER_EOS = 50257


def beam_search(engine, memory_slots, beam_slots, prompt, width=3, max_steps=128, eos=WHISPER_EOS,
                length_penalty=1.0, mask_special_023=True, stats=None):
    """memory_slots [U]; beam_slots [U][2*width] (distinct, reset here).
    Returns (list of token lists, normalised scores [U]); `stats` (a dict)
    receives the decoded row count."""
    mem = np.ascontiguousarray(memory_slots, dtype=np.int32)
    beams = np.ascontiguousarray(beam_slots, dtype=np.int32).reshape(mem.size, 2 * width)
    p = np.ascontiguousarray(prompt, dtype=np.int32)
    U = mem.size
    toks = np.zeros((U, max_steps), np.int32)
    lens = np.zeros(U, np.int32)
    scores = np.zeros(U, np.float32)
    cfg = BeamConfig(width, max_steps, eos, int(mask_special_023), length_penalty)
    rows = ctypes.c_longlong()
    call("ndl_beam_search", engine.handle, ctypes.byref(cfg), U, mem.ctypes.data, beams.ctypes.data, p.ctypes.data,
         p.size, toks.ctypes.data, lens.ctypes.data, scores.ctypes.data, ctypes.byref(rows))
    if stats is not None:
        stats["rows"] = rows.value
    return [list(map(int, toks[u, :lens[u]])) for u in range(U)], scores
