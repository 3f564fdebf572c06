"""The Needle-3 confidence head on the GPU: probe pooling over decoded
tokens (EngineCore.PoolTokensBatch, src/Needle/Engine.cs:2598-2650) and the
per-slot logit (ConfidenceLogitForSlot, :2702-2738), against the oracle's
scalar restatements.

Bar: pool max, sum, accumulators, cells and logits bit-exact (the online
softmax and the row softmax take MathF.Exp as the correctly rounded
exponential on both sides).  Batches mix decode rows, an
initial prefill run, fresh slots (peak -inf) and slots restored from a
snapshot.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_pool_update_and_logit_match_oracle(pkg, cuda, oracle):
    import torch

    from needle_cs_b200 import _native

    dev = torch.device("cuda:0")
    olib = oracle.lib()
    rng = np.random.default_rng(12)
    slots, dim, probes, layers, queries = 12, 256, 4, 3, 2
    pool_rows = (layers + 1) * probes
    probe_v = rng.normal(size=(pool_rows, dim)).astype(np.float32)
    cell = rng.normal(size=(slots, dim)).astype(np.float32)
    pmax = np.full((slots, pool_rows), -np.inf, np.float32)
    psum = np.zeros((slots, pool_rows), np.float32)
    pacc = np.zeros((slots, pool_rows, dim), np.float32)
    used = rng.permutation(slots)
    for s in used[:6]:  # slots with earlier tokens already pooled
        pmax[s] = rng.normal(size=pool_rows).astype(np.float32)
        psum[s] = rng.uniform(1, 5, pool_rows).astype(np.float32)
        pacc[s] = rng.normal(size=(pool_rows, dim)).astype(np.float32)
    snap_max, snap_sum = pmax + 0.5, psum * 2 + 0.1
    snap_acc = (pacc + 1).astype(np.float32)
    pending = np.zeros(slots, np.uint8)
    pending[used[:2]] = 1
    runs = [(used[0], 1), (used[1], 3), (used[2], 1), (used[6], 5), (used[7], 1)]
    row_slots = np.concatenate([np.full(n, s, np.int32) for s, n in runs])
    count = row_slots.size
    want = [a.copy() for a in (cell, pmax, psum, pacc)]
    d = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in dict(
        cell=cell, pmax=pmax, psum=psum, pacc=pacc, smax=snap_max, ssum=snap_sum, sacc=snap_acc, pend=pending,
        rs=row_slots, probe=probe_v).items()}
    for row in range(layers + 1):
        streams = rng.normal(size=(count, 4, dim)).astype(np.float32)
        initial = 1 if row == 0 else 0
        pend = pending if row == 0 else None  # the caller clears the flags after the first row
        olib.ndo_conf_pool_update(row, streams.ctypes.data, row_slots.ctypes.data, count, initial, probe_v.ctypes.data,
                                  probes, dim, pool_rows, want[0].ctypes.data, want[1].ctypes.data,
                                  want[2].ctypes.data, want[3].ctypes.data, snap_max.ctypes.data,
                                  snap_sum.ctypes.data, snap_acc.ctypes.data,
                                  pend.ctypes.data if pend is not None else None)
        ds = torch.from_numpy(streams).to(dev)
        _native.call("ndl_conf_pool_update", row, ds.data_ptr(), d["rs"].data_ptr(), count, initial,
                     d["probe"].data_ptr(), probes, dim, pool_rows, slots, d["cell"].data_ptr(), d["pmax"].data_ptr(),
                     d["psum"].data_ptr(), d["pacc"].data_ptr(), d["smax"].data_ptr(), d["ssum"].data_ptr(),
                     d["sacc"].data_ptr(), d["pend"].data_ptr() if pend is not None else None, None)
    got = [d[k].cpu().numpy() for k in ("cell", "pmax", "psum", "pacc")]
    assert np.array_equal(got[0], want[0])
    for g, w in zip(got[1:], want[1:]):
        fin = np.isfinite(w)
        assert np.array_equal(np.isfinite(g), fin)
        assert np.array_equal(g[fin], w[fin])

    # the logit of every touched slot, from the pools the oracle made
    gain = rng.uniform(0.5, 1.5, pool_rows).astype(np.float32)
    qv = rng.normal(size=(queries, dim)).astype(np.float32)
    rb = rng.normal(size=(queries, pool_rows)).astype(np.float32) * 0.1
    proj = rng.normal(size=queries * dim).astype(np.float32) * 0.05
    listed = np.array([s for s, _ in runs], np.int32)
    dsum, dacc = torch.from_numpy(want[2]).to(dev), torch.from_numpy(want[3]).to(dev)
    t = {k: torch.from_numpy(v).to(dev) for k, v in dict(l=listed, g=gain, q=qv, rb=rb, p=proj).items()}
    logits = torch.empty(listed.size, device=dev)
    pooled = torch.empty((listed.size, queries, dim), device=dev)
    _native.call("ndl_conf_logit", t["l"].data_ptr(), listed.size, dsum.data_ptr(), dacc.data_ptr(), pool_rows, dim,
                 t["g"].data_ptr(), t["q"].data_ptr(), t["rb"].data_ptr(), 0.25, t["p"].data_ptr(), queries,
                 logits.data_ptr(), pooled.data_ptr(), None)
    gl, gp = logits.cpu().numpy(), pooled.cpu().numpy()
    for r, s in enumerate(listed):
        wp = np.zeros((queries, dim), np.float32)
        wl = olib.ndo_conf_logit(want[2][s].ctypes.data, want[3][s].ctypes.data, pool_rows, dim, gain.ctypes.data,
                                 qv.ctypes.data, rb.ctypes.data, 0.25, proj.ctypes.data, queries, wp.ctypes.data)
        assert np.float32(gl[r]) == np.float32(wl), (r, gl[r], wl)
        assert np.array_equal(gp[r], wp)
