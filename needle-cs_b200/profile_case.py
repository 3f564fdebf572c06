"""Small, self-contained cases for kernel captures under a profiler.

    python needle-cs_b200/profile_case.py attention
    python needle-cs_b200/profile_case.py gemm M N K

attention: a 2-layer synthetic decoder with the cfg5 batch shape (512 rows,
8 heads, per-session prefixes uniform in [64, 1024] positions), so each
attention launch has the full-size launch shape while the engine holds about
1.3 GB of KV pages instead of 12 layers' worth.  Runs 4 profiled steps and
prints the per-class device times.

gemm M N K: five calls of the I8G32 linear (ndl_matmul_i8g32) on random
int8 activations [M,K] and weights [N,K] with fp16 group scales; M >= 64
runs the tcgen05 GEMM, smaller M the GEMV.
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


def gemm_case(m, n, k, calls=5):
    import torch

    entry.load_package()
    import importlib

    ops = importlib.import_module("needle_cs_b200.ops")
    dev = torch.device("cuda:0")
    q = torch.randint(-128, 128, (m, k), dtype=torch.int8, device=dev)
    sa = torch.rand(m, device=dev) * 0.01
    w = torch.randint(-127, 128, (n, k), dtype=torch.int8, device=dev)
    sw = torch.full((n, k // 32), 0x2000, dtype=torch.int16, device=dev)
    y = torch.empty((m, n), device=dev)
    for _ in range(calls):
        ops.matmul_i8g32(q, sa, w, sw, y=y)
    torch.cuda.synchronize()
    print("gemm", m, n, k, "ok")


if __name__ == "__main__":
    case = sys.argv[1] if len(sys.argv) > 1 else "attention"
    if case == "attention":
        attention_case()
    elif case == "gemm":
        gemm_case(*(int(v) for v in sys.argv[2:5]))
    else:
        raise SystemExit(f"unknown case {case!r}")
