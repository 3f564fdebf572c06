"""The Engram block of a loaded model on the GPU (ndl_engram_apply), against
the oracle's scalar chain of ApplyEngramBatch (src/Needle/Engine.cs:2405-2469):
the row hash, GatherRow of each table row (zeros for a row the n-gram does not
reach yet), Quant.FakeA8, Quant.Prepare at 2 bits, the key and value CQ
matmuls, the dilated conv over the slot history and the gated residual add.

Bar: the new slot histories and the residual bit-exact (every step, the
gate's sigmoid included, takes the scalar code's operations one rounding at a
time; MathF.Exp is the correctly rounded exponential on both sides).  The batch mixes decode rows with prefill runs, and slots too
short for an n-gram.  Two calls in a row check that the workspace carries
nothing from one call to the next.
"""
import numpy as np
import pytest

from cact_support import Archive

pytestmark = pytest.mark.gpu

GEOMETRY = dict(dim=512, engram_sub=128, engram_tables=4, engram_slots=97, orders=[2, 3], engram_dilation=2)


def _oracle_block(oracle, m, a, tokens, row_slots, slot_length, slot_prev, hist, x, residual):
    g = m.info
    lib = oracle.lib()
    count, dim, tables = row_slots.size, g["dim"], g["engram_tables"]
    heads = tables // g["order_count"]
    orders = np.array(g["orders"], np.int32)
    rows = np.zeros((count, tables), np.int32)
    lib.ndo_engram_hash(tokens.ctypes.data, row_slots.ctypes.data, count, slot_length.ctypes.data,
                        slot_prev.ctypes.data, orders.ctypes.data, orders.size, heads, g["engram_slots"],
                        rows.ctypes.data)
    rec = {(r[0], r[1]): r[6] for r in a.records}
    tab = m.tensor("site.tables", 0)
    _, codes, norms, nrows, cols, bits = rec[("site.tables", 0)]
    codes, norms = codes.reshape(nrows, -1), norms.reshape(nrows, -1)
    levels = np.array(tab.book.contents.levels, np.float32)
    e = np.zeros((count, dim), np.float32)
    for t in range(count):
        for table in range(tables):
            if rows[t, table] >= 0:
                e[t, table * cols:(table + 1) * cols] = oracle.gather_row_cq(codes, norms, levels, bits,
                                                                             int(rows[t, table]))
        lib.ndo_fake_a8(e[t].ctypes.data, dim)
    vals, sc, off, _ = oracle.prepare_cq(e, 2)
    book2 = oracle.codebook(a.levels[0:4], 4)

    def matmul(role):
        _, c, n, r, _, _ = rec[(role, 0)]
        return oracle.matmul_rows_cq(c.reshape(r, -1), n.reshape(r, -1), book2, 2, vals, sc, off)

    key, value = matmul("site.key"), matmul("site.value")
    taps = np.ascontiguousarray(m.host("site.taps")[:4 * dim])
    conv = np.zeros((count, dim), np.float32)
    hout = hist.copy()
    lib.ndo_engram_conv(hist.ctypes.data, value.ctypes.data, row_slots.ctypes.data, count, taps.ctypes.data,
                        g["engram_dilation"], dim, conv.ctypes.data, hout.ctypes.data)
    res = residual.copy()
    for t in range(count):
        lib.ndo_engram_gate(x[t].ctypes.data, key[t].ctypes.data, conv[t].ctypes.data, dim, res[t].ctypes.data)
    return rows, conv, hout, res


def test_engram_block_matches_the_scalar_chain(pkg, cuda, oracle):
    import importlib

    import torch

    from needle_cs_b200 import _native

    cact = importlib.import_module("needle_cs_b200.model")
    a = Archive(seed=31, geometry=GEOMETRY).standard()
    m = cact.Model.from_bytes(a.build(), device=0)
    try:
        rng = np.random.default_rng(32)
        slots, dim = 12, GEOMETRY["dim"]
        lengths = [1, 1, 3, 1, 4, 1]
        picks = rng.permutation(slots)[:len(lengths)]
        row_slots = np.concatenate([np.full(n, s, np.int32) for s, n in zip(picks, lengths)])
        count = row_slots.size
        tokens = rng.integers(0, 50000, count).astype(np.int32)
        slot_length = rng.integers(0, 6, slots).astype(np.int32)
        slot_length[picks[:2]] = 0  # n-grams that do not fit yet
        slot_prev = rng.integers(0, 50000, (slots, 2)).astype(np.int32)
        hist = rng.normal(size=(slots, 9, dim)).astype(np.float32)
        x = rng.normal(size=(count, dim)).astype(np.float32)
        residual = rng.normal(size=(count, dim)).astype(np.float32)
        rows, conv, want_hist, want_res = _oracle_block(oracle, m, a, tokens, row_slots, slot_length, slot_prev, hist,
                                                        x, residual)
        assert (rows == -1).any() and (rows >= 0).any()
        dev = torch.device("cuda:0")
        d = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in dict(
            tok=tokens, rs=row_slots, sl=slot_length, sp=slot_prev, hist=hist, x=x).items()}
        need = _native.lib().ndl_engram_workspace(m._h, count)
        assert need > 0
        ws = torch.empty(need, dtype=torch.uint8, device=dev)
        for call in range(3):  # two calls through the C ABI on one workspace, one through the mirror
            res = torch.from_numpy(residual).to(dev)
            hout = d["hist"].clone()
            if call < 2:
                _native.call("ndl_engram_apply", m._h, 0, d["tok"].data_ptr(), d["rs"].data_ptr(), count,
                             d["sl"].data_ptr(), d["sp"].data_ptr(), slots, d["hist"].data_ptr(), hout.data_ptr(),
                             d["x"].data_ptr(), res.data_ptr(), ws.data_ptr(), need, None)
            else:
                m.apply_engram(0, d["tok"], d["rs"], d["sl"], d["sp"], d["hist"], hout, d["x"], res)
            torch.cuda.synchronize()
            assert np.array_equal(hout.cpu().numpy().view(np.uint32), want_hist.view(np.uint32))
            got = res.cpu().numpy()
            assert np.array_equal(got.view(np.uint32), want_res.view(np.uint32)), np.abs(got - want_res).max()
        assert np.abs(want_res - residual).max() > 0.01  # the block changes the residual
        with pytest.raises(_native.NeedleError, match="workspace"):
            _native.call("ndl_engram_apply", m._h, 0, d["tok"].data_ptr(), d["rs"].data_ptr(), count,
                         d["sl"].data_ptr(), d["sp"].data_ptr(), slots, d["hist"].data_ptr(), hout.data_ptr(),
                         d["x"].data_ptr(), res.data_ptr(), ws.data_ptr(), need - 1, None)
    finally:
        m.close()
