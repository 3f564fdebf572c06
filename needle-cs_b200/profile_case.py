"""Small, self-contained cases for kernel captures under a profiler.

    python needle-cs_b200/profile_case.py attention

attention: a 2-layer synthetic decoder with the cfg5 batch shape (512 rows,
8 heads, per-session prefixes uniform in [64, 1024] positions), so each
attention launch has the full-size launch shape while the engine holds about
1.3 GB of KV pages instead of 12 layers' worth.  Runs 4 profiled steps and
prints the per-class device times.
"""
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import __graft_entry__ as entry  # noqa: E402


def attention_case(steps=4, rows=512, seed=5):
    entry.load_package()
    from needle_cs_b200.engine import BatchedEngine, SyntheticDecoder

    eng = BatchedEngine(SyntheticDecoder(layers=2, seed=1), slots=rows, context_length=1088, chunk_size=512,
                        max_heads=rows)
    lengths = np.random.default_rng(seed).integers(64, 1025, rows)
    for j in range(rows):
        eng.fill_synthetic(j, int(lengths[j]), seed, j)
    tokens = np.random.default_rng(seed + 1).integers(0, 8192, rows).astype(np.int32)
    order = np.arange(rows, dtype=np.int32)
    eng.profile(True)
    for _ in range(steps):
        eng.forward_batch(tokens, order, order)
        tokens = eng.sample_argmax()
    eng.sync()
    prof = eng.profile_read()
    eng.close()
    print({k: (round(v[0], 3), v[1]) for k, v in prof.items()})


if __name__ == "__main__":
    case = sys.argv[1] if len(sys.argv) > 1 else "attention"
    if case != "attention":
        raise SystemExit(f"unknown case {case!r}")
    attention_case()
