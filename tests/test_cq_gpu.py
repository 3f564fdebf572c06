"""CQ weights on the GPU: Quant.Prepare (src/Needle/Quant.cs:471-484) and
MatMulRows on CQ matrices (Scalar.MatMulRows, src/Needle/Scalar.cs:146-192),
through the KernelTable-signature exports (slots 0 and 1, host pointers) and
the device-pointer entry points.

Bars: prepared values, scales and offsets equal the oracle's scalar branch
bit for bit; y equals the oracle's MatMulRows bit for bit; entries outside
[rowStart, rowEnd) and the stride padding stay untouched; bad shapes fail with
NDL_ERR_INVALID_ARG.  Shapes follow the reference's MatMul conformance cases
(KernelConformanceTests.cs:51-185) plus decode-sized matrices.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


class KtCodebook(ctypes.Structure):
    _fields_ = [("levels", ctypes.c_float * 16), ("bytes", ctypes.c_uint8 * 32), ("byte_scale", ctypes.c_float)]


class KtCq(ctypes.Structure):
    _fields_ = [("indices", ctypes.c_void_p), ("norms", ctypes.c_void_p), ("book", ctypes.c_void_p),
                ("rows", ctypes.c_int), ("cols", ctypes.c_int), ("bits", ctypes.c_int)]


class KtActivations(ctypes.Structure):
    _fields_ = [("values", ctypes.c_void_p), ("scales", ctypes.c_void_p), ("offsets", ctypes.c_void_p),
                ("cols", ctypes.c_int), ("groups", ctypes.c_int), ("stride", ctypes.c_int)]


@pytest.fixture(scope="module")
def lib(pkg, cuda):
    from needle_cs_b200 import _native

    so = _native.lib()
    so.ndl_kt_matmul_rows.restype = None
    so.ndl_kt_matmul_rows.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_int]
    so.ndl_kt_prepare.restype = None
    so.ndl_kt_prepare.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return so


def _weights(oracle, seed, bits, rows, cols):
    """ConformanceWeights-style CQ matrix: jittered levels, random index bytes
    (with extremes), norms in [0.2, 2.0)."""
    rng = oracle.XorShift64(seed)
    count = 4 if bits == 2 else 16
    levels = np.zeros(16, np.float32)
    for i in range(count):
        levels[i] = np.float32((i - (count - 1) / 2) * 0.4) + np.float32(rng.next_float(0.05))
    book = oracle.codebook(levels, count)
    row_bytes = cols * bits // 8
    fill = oracle.XorShift64(seed ^ 0x5BD1E995)
    idx = fill.fill_bytes(rows * row_bytes, True)[:rows * row_bytes].reshape(rows, row_bytes)
    groups = cols // 128
    norms = np.array([oracle.lib().ndo_half_bits(np.float32(0.2 + (fill.next() % 1000) * 0.0018))
                      for _ in range(rows * groups)], np.uint16).reshape(rows, groups)
    return book, idx, norms


def _x(oracle, seed, tokens, cols):
    x = oracle.XorShift64(seed ^ 0x243F6A88).fill_edges(tokens * cols, 3.0)[:tokens * cols].reshape(tokens, cols)
    if tokens and cols >= 256:
        x[0, 128:256] = 0.0  # an all-zero group: peak 0, scale 1
    return np.ascontiguousarray(x)


def _kt_prepare(lib, x, bits, stride):
    tokens, cols = x.shape
    vals = np.full((tokens, cols), 99, np.int8)
    sc = np.full((tokens, stride), -7.0, np.float32)
    off = np.full((tokens, stride), -7.0, np.float32)
    act = KtActivations(vals.ctypes.data, sc.ctypes.data, off.ctypes.data, cols, cols // 128, stride)
    lib.ndl_kt_prepare(x.ctypes.data, tokens, cols, bits, ctypes.byref(act))
    return vals, sc, off


@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("tokens,cols", [(1, 128), (2, 768), (5, 384), (3, 4096), (16, 512), (20, 1024)])
def test_prepare_matches_oracle(lib, oracle, bits, tokens, cols):
    x = _x(oracle, 0x1234 + cols, tokens, cols)
    want_v, want_s, want_o, stride = oracle.prepare_cq(x, bits)
    vals, sc, off = _kt_prepare(lib, x, bits, stride)
    groups = cols // 128
    assert np.array_equal(vals, want_v)
    assert np.array_equal(sc[:, :groups].view(np.uint32), want_s[:, :groups].view(np.uint32))
    assert np.array_equal(off[:, :groups].view(np.uint32), want_o[:, :groups].view(np.uint32))
    assert (sc[:, groups:] == -7.0).all() and (off[:, groups:] == -7.0).all()  # padding untouched


MATMUL_CASES = [  # (bits, rows, cols, tokens): the conformance shapes, then decode-sized ones
    (2, 5, 768, 1), (2, 5, 768, 3), (4, 7, 384, 5), (2, 3, 128, 8), (4, 97, 768, 3), (2, 5, 768, 0),
    (2, 2048, 512, 1), (4, 2048, 512, 16), (2, 512, 4096, 2), (4, 1000, 1024, 20),
    # many tokens (8-token blocks, a ragged last block) and long rows: the group-split kernel
    (2, 600, 768, 64), (4, 40, 3072, 33), (2, 24, 8192, 9),
    # enough 16-row tiles for the warp-per-tile kernel (<= 16 tokens)
    (2, 20000, 256, 5), (4, 19000, 128, 16),
]


@pytest.mark.parametrize("bits,rows,cols,tokens", MATMUL_CASES)
def test_matmul_rows_matches_oracle(lib, oracle, bits, rows, cols, tokens):
    book, idx, norms = _weights(oracle, 0x1234 + rows, bits, rows, cols)
    x = _x(oracle, 0x9ABC + rows, tokens, cols)
    vals, sc, off, stride = oracle.prepare_cq(x, bits) if tokens else (
        np.zeros((0, cols), np.int8), np.zeros((0, 8), np.float32), np.zeros((0, 8), np.float32), 8)
    ldy = rows + 3
    want = np.full((tokens, ldy), 5.0, np.float32)
    if tokens:
        want[:, :rows] = oracle.matmul_rows_cq(idx, norms, book, bits, vals, sc, off)
    kbook = KtCodebook.from_buffer_copy(bytes(book))
    w = KtCq(idx.ctypes.data, norms.ctypes.data, ctypes.addressof(kbook), rows, cols, bits)
    act = KtActivations(vals.ctypes.data, sc.ctypes.data, off.ctypes.data, cols, cols // 128, stride)
    got = np.full((max(tokens, 1), ldy), 5.0, np.float32)
    lib.ndl_kt_matmul_rows(ctypes.byref(w), ctypes.byref(act), tokens, got.ctypes.data, ldy, 0, rows)
    assert np.array_equal(got[:tokens].view(np.uint32), want.view(np.uint32))
    assert (got[:, rows:] == 5.0).all()


def test_matmul_rows_range_leaves_other_rows(lib, oracle):
    """Golden range case (KernelConformanceTests 'range_odd': seed 0x9ABC, 2-bit, 8 x 128, rows 3..7)."""
    bits, rows, cols, tokens, r0, r1 = 2, 8, 128, 3, 3, 7
    book, idx, norms = _weights(oracle, 0x9ABC, bits, rows, cols)
    vals, sc, off, stride = oracle.prepare_cq(_x(oracle, 0x9ABC, tokens, cols), bits)
    want = oracle.matmul_rows_cq(idx, norms, book, bits, vals, sc, off, r0, r1, y=np.full((tokens, rows), 5.0,
                                                                                        np.float32))
    kbook = KtCodebook.from_buffer_copy(bytes(book))
    w = KtCq(idx.ctypes.data, norms.ctypes.data, ctypes.addressof(kbook), rows, cols, bits)
    act = KtActivations(vals.ctypes.data, sc.ctypes.data, off.ctypes.data, cols, 1, stride)
    got = np.full((tokens, rows), 5.0, np.float32)
    lib.ndl_kt_matmul_rows(ctypes.byref(w), ctypes.byref(act), tokens, got.ctypes.data, rows, r0, r1)
    assert np.array_equal(got, want)
    assert (got[:, :r0] == 5.0).all() and (got[:, r1:] == 5.0).all()


def test_device_entry_points(pkg, oracle):
    """ndl_cq_prepare + ndl_cq_matmul on device memory equal the oracle."""
    import torch

    from needle_cs_b200 import NeedleError, _native

    dev = torch.device("cuda:0")
    bits, rows, cols, tokens = 4, 3000, 2048, 4
    book, idx, norms = _weights(oracle, 77, bits, rows, cols)
    x = _x(oracle, 78, tokens, cols)
    want_v, want_s, want_o, stride = oracle.prepare_cq(x, bits)
    want_y = oracle.matmul_rows_cq(idx, norms, book, bits, want_v, want_s, want_o)
    dx = torch.from_numpy(x).to(dev)
    dv = torch.zeros((tokens, cols), dtype=torch.int8, device=dev)
    ds = torch.zeros((tokens, stride), dtype=torch.float32, device=dev)
    do = torch.zeros((tokens, stride), dtype=torch.float32, device=dev)
    _native.call("ndl_cq_prepare", dx.data_ptr(), tokens, cols, bits, dv.data_ptr(), ds.data_ptr(), do.data_ptr(),
                 stride, None)
    di = torch.from_numpy(idx).to(dev)
    dn = torch.from_numpy(norms.view(np.int16)).to(dev)
    dy = torch.zeros((tokens, rows), dtype=torch.float32, device=dev)
    table = (ctypes.c_uint8 * 16).from_buffer_copy(bytes(book.bytes)[:16])
    _native.call("ndl_cq_matmul", di.data_ptr(), dn.data_ptr(), ctypes.addressof(table), book.byte_scale, rows, cols,
                 bits, dv.data_ptr(), ds.data_ptr(), do.data_ptr(), stride, tokens, dy.data_ptr(), rows, 0, rows,
                 None)
    torch.cuda.synchronize()
    assert np.array_equal(dv.cpu().numpy(), want_v)
    assert np.array_equal(ds.cpu().numpy(), want_s) and np.array_equal(do.cpu().numpy(), want_o)
    assert np.array_equal(dy.cpu().numpy().view(np.uint32), want_y.view(np.uint32))
    with pytest.raises(NeedleError) as e:  # cols not a multiple of 128
        _native.call("ndl_cq_matmul", di.data_ptr(), dn.data_ptr(), ctypes.addressof(table), book.byte_scale, rows,
                     100, bits, dv.data_ptr(), ds.data_ptr(), do.data_ptr(), stride, tokens, dy.data_ptr(), rows, 0,
                     rows, None)
    assert e.value.status == 100


@pytest.mark.parametrize("bits,rows,cols", [(2, 6, 128), (4, 9, 768), (2, 300, 2048), (4, 33, 4096)])
def test_gather_row_matches_oracle(lib, oracle, bits, rows, cols):
    """GatherRow (slot 2) and the batched device entry point equal the oracle's
    DecodeRow + Hadamard bit for bit."""
    import torch

    from needle_cs_b200 import _native

    lib.ndl_kt_gather_row.restype = None
    lib.ndl_kt_gather_row.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    book, idx, norms = _weights(oracle, 0x4321 + rows, bits, rows, cols)
    levels = np.frombuffer(bytes(book)[:64], np.float32)
    kbook = KtCodebook.from_buffer_copy(bytes(book))
    w = KtCq(idx.ctypes.data, norms.ctypes.data, ctypes.addressof(kbook), rows, cols, bits)
    picks = sorted({0, rows - 1, rows // 2, 1 % rows})
    for row in picks:
        got = np.full(cols, 7.0, np.float32)
        lib.ndl_kt_gather_row(ctypes.byref(w), row, got.ctypes.data)
        want = oracle.gather_row_cq(idx, norms, levels, bits, row)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), row
    dev = torch.device("cuda:0")
    ids = np.array(picks[::-1] + picks, np.int32)  # reordered and repeated rows
    di, dn = torch.from_numpy(idx).to(dev), torch.from_numpy(norms.view(np.int16)).to(dev)
    dids = torch.from_numpy(ids).to(dev)
    out = torch.zeros((ids.size, cols), dtype=torch.float32, device=dev)
    lv = np.ascontiguousarray(levels)
    _native.call("ndl_cq_gather_rows", di.data_ptr(), dn.data_ptr(), lv.ctypes.data, rows, cols, bits,
                 dids.data_ptr(), ids.size, out.data_ptr(), None)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for r, row in enumerate(ids):
        assert np.array_equal(got[r], oracle.gather_row_cq(idx, norms, levels, bits, int(row))), (r, row)
