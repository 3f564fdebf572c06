"""Engram, the Needle-3 n-gram memory, on the GPU: the row hash
(EngramHashRowsBatch, src/Needle/Engine.cs:2652-2681), the causal conv over
the slot history and the residual gate (ApplyEngramBatch, :2405-2469),
against the oracle's scalar restatements.

Bar: hash rows, conv outputs, the new slot histories and the gated residual
bit-exact (the gate's sigmoid takes the correctly rounded exponential on
both sides).  Batches mix decode rows (runs of one) with prefill runs of
several tokens of one slot, including slots too short for an n-gram.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _runs(rng, slots, lengths):
    """row_slots for runs of the given lengths over distinct slots."""
    picks = rng.permutation(slots)[:len(lengths)]
    return np.concatenate([np.full(n, s, np.int32) for s, n in zip(picks, lengths)])


@pytest.fixture(scope="module")
def dev(pkg, cuda):
    import torch

    return torch.device("cuda:0")


def _t(a, dev):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def test_engram_hash_matches_oracle(dev, oracle):
    from needle_cs_b200 import _native

    rng = np.random.default_rng(4)
    slots, heads, engram_slots = 40, 4, 65521
    orders = np.array([2, 3], np.int32)
    row_slots = _runs(rng, slots, [1, 1, 5, 1, 3, 12, 1, 2])
    count = row_slots.size
    tokens = rng.integers(0, 50000, count).astype(np.int32)
    slot_length = rng.integers(0, 6, slots).astype(np.int32)  # 0 and 1: n-grams that do not fit yet
    slot_length[row_slots[:2]] = 0
    slot_prev = rng.integers(0, 50000, (slots, 2)).astype(np.int32)
    tables = orders.size * heads
    want = np.zeros((count, tables), np.int32)
    olib = oracle.lib()
    olib.ndo_engram_hash(tokens.ctypes.data, row_slots.ctypes.data, count, slot_length.ctypes.data,
                         slot_prev.ctypes.data, orders.ctypes.data, orders.size, heads, engram_slots,
                         want.ctypes.data)
    d = {k: _t(v, dev) for k, v in dict(tok=tokens, rs=row_slots, sl=slot_length, sp=slot_prev).items()}
    import torch

    rows = torch.empty((count, tables), dtype=torch.int32, device=dev)
    _native.call("ndl_engram_hash", d["tok"].data_ptr(), d["rs"].data_ptr(), count, d["sl"].data_ptr(),
                 d["sp"].data_ptr(), slots, orders.ctypes.data, orders.size, heads, engram_slots, rows.data_ptr(), None)
    got = rows.cpu().numpy()
    assert np.array_equal(got, want)
    assert (want == -1).any() and (want >= 0).any()


@pytest.mark.parametrize("dilation", [1, 2, 3])
def test_engram_conv_matches_oracle(dev, oracle, dilation):
    import torch

    from needle_cs_b200 import _native

    rng = np.random.default_rng(10 + dilation)
    slots, dim = 16, 384
    row_slots = _runs(rng, slots, [1, 4, 1, 11, 2, 1])
    count = row_slots.size
    hist = rng.normal(size=(slots, 9, dim)).astype(np.float32)
    values = rng.normal(size=(count, dim)).astype(np.float32)
    taps = rng.normal(size=(4, dim)).astype(np.float32)
    want_out = np.zeros((count, dim), np.float32)
    want_hist = hist.copy()
    oracle.lib().ndo_engram_conv(hist.ctypes.data, values.ctypes.data, row_slots.ctypes.data, count,
                                 taps.ctypes.data, dilation, dim, want_out.ctypes.data, want_hist.ctypes.data)
    dh, dv, dr, dt = _t(hist, dev), _t(values, dev), _t(row_slots, dev), _t(taps, dev)
    out = torch.empty((count, dim), device=dev)
    hout = dh.clone()
    _native.call("ndl_engram_conv", dh.data_ptr(), dv.data_ptr(), dr.data_ptr(), count, slots, dt.data_ptr(),
                 dilation, dim, out.data_ptr(), hout.data_ptr(), None)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want_out.view(np.uint32))
    assert np.array_equal(hout.cpu().numpy().view(np.uint32), want_hist.view(np.uint32))


@pytest.mark.parametrize("dim", [768, 130])  # the CTA-per-row kernel; a width it does not take
def test_engram_gate_matches_oracle(dev, oracle, dim):
    import torch

    from needle_cs_b200 import _native

    rng = np.random.default_rng(5)
    count = 37
    x = rng.normal(size=(count, dim)).astype(np.float32)
    key = (x * 0.5 + rng.normal(size=(count, dim))).astype(np.float32)
    v = rng.normal(size=(count, dim)).astype(np.float32)
    res = rng.normal(size=(count, dim)).astype(np.float32)
    want = res.copy()
    for t in range(count):
        oracle.lib().ndo_engram_gate(x[t].ctypes.data, key[t].ctypes.data, v[t].ctypes.data, dim,
                                     want[t].ctypes.data)
    dres, dx, dk, dv = _t(res, dev), _t(x, dev), _t(key, dev), _t(v, dev)  # held until the kernel has run
    _native.call("ndl_engram_gate", dx.data_ptr(), dk.data_ptr(), dv.data_ptr(), count, dim, dres.data_ptr(), None)
    torch.cuda.synchronize()
    got = dres.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), np.abs(got - want).max()
    assert np.abs(want - res).max() > 0.1  # the gate is open enough to matter
