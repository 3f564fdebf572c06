"""Data-parallel placement across ranks, on the CPU with gloo (world size 2):
the benchmark's session partition (global session i -> rank i mod N, no
collective on the data path) and its timing plumbing (barrier, max over
ranks).  The GPU path runs the same code with NCCL."""
import importlib.util
import os
import socket

import numpy as np
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _worker(rank, world, port, out):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        b = _bench()
        wl = b.DecodeWorkload("cfg5")
        gids, lengths, _ = wl.global_layout(rank, world)
        b.barrier(world)
        t = b.max_over_ranks(float(10 + rank), world)
        gathered = [None] * world
        dist.all_gather_object(gathered, (list(map(int, gids)), list(map(int, lengths)), t))
        if rank == 0:
            out.put(gathered)
    finally:
        dist.destroy_process_group()


def test_sessions_partition_round_robin_and_max_over_ranks():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    gathered = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (g0, l0, t0), (g1, l1, t1) = gathered
    assert t0 == t1 == 11.0                                # max over ranks
    assert len(g0) == len(g1) == 1024                      # 1024 sessions per GPU
    assert set(g0).isdisjoint(g1)
    assert sorted(g0 + g1) == list(range(2048))            # every global session once
    assert all(g % 2 == 0 for g in g0) and all(g % 2 == 1 for g in g1)
    # a session's KV length is a function of its global id only
    wl = _bench().DecodeWorkload("cfg5")
    lengths = np.random.default_rng(wl.seed).integers(wl.lo, wl.hi + 1, size=2 * wl.sessions)
    assert list(lengths[g0]) == l0 and list(lengths[g1]) == l1
