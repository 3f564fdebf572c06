"""The .cact loader's upload on the GPU: ndl_model_load with device 0.

Every uploaded tensor is read back through its device address and compared
with the archive: CQ codes and norms byte for byte, dense tensors bit for bit
with the host rule, permutations exactly.  The probe heads' decoded rows
(Reader.Rows, src/Needle/Model.cs:220-225) are compared with the oracle's
GatherRow bit for bit.  The model's tensors then drive the device kernels
directly, each checked bit for bit against the oracle:
 * an embedding gather (ndl_cq_gather_rows on "embedding");
 * a CQ matmul (ndl_cq_matmul on "layer.gate" 1 with the model's codebook);
 * the confidence head (ndl_conf_pool_update and ndl_conf_logit on the
   probe head's tensors), bit for bit as well (MathF.Exp is the correctly
   rounded exponential on both sides).
"""
import ctypes

import numpy as np
import pytest

from cact_support import Archive

pytestmark = pytest.mark.gpu


class _DeviceArray:
    """A raw device address as a CUDA array (the tests only read it; torch
    takes no read-only flag)."""

    def __init__(self, ptr, n, typestr):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3}


def _read(ptr, n, typestr, np_dtype):
    import torch

    return torch.as_tensor(_DeviceArray(ptr, n, typestr), device="cuda:0").cpu().numpy().astype(np_dtype, copy=False)


@pytest.fixture(scope="module")
def loaded(pkg, cuda):
    import importlib

    cact = importlib.import_module("needle_cs_b200.model")
    a = Archive(seed=21).standard(probe_codes=(2,))
    m = cact.Model.from_bytes(a.build(), device=0)
    yield cact, a, m
    m.close()


def test_every_tensor_is_uploaded(loaded):
    cact, a, m = loaded
    info = m.info
    assert info["device"] == 0 and info["device_bytes"] > 0
    for role, index, _, _, _, _, exp in a.records:
        if role == "tokenizer":
            continue
        t = m.tensor(role, index)
        if exp[0] == "cq":
            codes, norms = exp[1], exp[2]
            assert np.array_equal(_read(t.indices, codes.size, "|u1", np.uint8), codes)
            assert np.array_equal(_read(t.norms, norms.size, "<i2", np.int16).view(np.uint16), norms)
        elif exp[0] == "perm":
            assert np.array_equal(_read(t.permutation, t.count, "<i4", np.int32), exp[1])
        else:
            got = _read(t.values, t.count, "<f4", np.float32)
            assert np.array_equal(got.view(np.uint32), m.host(role, index).view(np.uint32)), (role, index)


def test_probe_rows_are_decoded_like_gather_row(loaded, oracle):
    cact, a, m = loaded
    for role in ("probe.probe_vectors", "probe.query_vectors", "probe.projection"):
        t = m.tensor(role, 0)
        assert t.kind == cact.CQ_ROWS
        exp = next(r[6] for r in a.records if r[0] == role)
        codes = exp[1].reshape(t.rows, -1)
        norms = exp[2].reshape(t.rows, -1)
        levels = np.array(t.book.contents.levels, np.float32)
        want = np.stack([oracle.gather_row_cq(codes, norms, levels, t.bits, r) for r in range(t.rows)])
        got = _read(t.values, t.rows * t.cols, "<f4", np.float32).reshape(t.rows, t.cols)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), role


def test_model_tensors_drive_the_kernels(loaded, oracle):
    import torch

    from needle_cs_b200 import _native

    cact, a, m = loaded
    emb = m.tensor("embedding", 0)
    ids = np.array([0, 7, 255, 128, 7], np.int32)
    d_ids = torch.from_numpy(ids).cuda()
    out = torch.empty((ids.size, emb.cols), device="cuda:0")
    _native.call("ndl_cq_gather_rows", emb.indices, emb.norms, ctypes.addressof(emb.book.contents.levels), emb.rows,
                 emb.cols, emb.bits, d_ids.data_ptr(), ids.size, out.data_ptr(), None)
    exp = next(r[6] for r in a.records if r[0] == "embedding")
    codes, norms = exp[1].reshape(emb.rows, -1), exp[2].reshape(emb.rows, -1)
    levels = np.array(emb.book.contents.levels, np.float32)
    want = np.stack([oracle.gather_row_cq(codes, norms, levels, emb.bits, int(i)) for i in ids])
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))

    w = m.tensor("layer.gate", 1)
    x = np.random.default_rng(3).normal(size=(5, w.cols)).astype(np.float32)
    vals, sc, off, stride = oracle.prepare_cq(x, w.bits)
    dv, ds, do = (torch.from_numpy(v).cuda() for v in (vals, sc, off))
    y = torch.empty((5, w.rows), device="cuda:0")
    book = w.book.contents
    _native.call("ndl_cq_matmul", w.indices, w.norms, ctypes.addressof(book.bytes), float(book.byte_scale), w.rows,
                 w.cols, w.bits, dv.data_ptr(), ds.data_ptr(), do.data_ptr(), stride, 5, y.data_ptr(), w.rows, 0,
                 w.rows, None)
    exp = next(r[6] for r in a.records if r[0] == "layer.gate" and r[1] == 1)
    obook = oracle.codebook(a.levels[0:4], 4)
    want = oracle.matmul_rows_cq(exp[1].reshape(w.rows, -1), exp[2].reshape(w.rows, -1), obook, w.bits, vals, sc, off)
    torch.cuda.synchronize()
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_confidence_head_runs_on_model_weights(loaded, oracle):
    """The n7 kernels (ndl_conf_pool_update, ndl_conf_logit) fed by the
    model's confidence head: decoded probe, query and projection rows, gain,
    row bias and bias, against the oracle on the same tensors."""
    import torch

    from needle_cs_b200 import _native

    cact, a, m = loaded
    info = m.info
    h = info["confidence_head"]
    assert h == 0
    probes_t, query_t, proj_t = (m.tensor(r, h) for r in ("probe.probe_vectors", "probe.query_vectors",
                                                          "probe.projection"))
    dim, layers = info["dim"], info["layers"]
    pool_rows, queries = probes_t.rows, query_t.rows
    probes = pool_rows // (layers + 1)
    rows_of = lambda t: _read(t.values, t.rows * t.cols, "<f4", np.float32).reshape(t.rows, t.cols)
    probe_v, qv, proj = rows_of(probes_t), rows_of(query_t), rows_of(proj_t).reshape(-1)
    gain, rb, bias = m.host("probe.gain", h), m.host("probe.row_bias", h), float(m.host("probe.bias", h)[0])
    rng = np.random.default_rng(41)
    slots = 6
    row_slots = np.array([3, 3, 1, 4, 4, 4], np.int32)
    count = row_slots.size
    cell = np.zeros((slots, dim), np.float32)
    pmax = np.full((slots, pool_rows), -np.inf, np.float32)
    psum = np.zeros((slots, pool_rows), np.float32)
    pacc = np.zeros((slots, pool_rows, dim), np.float32)
    want = [x.copy() for x in (cell, pmax, psum, pacc)]
    dev = torch.device("cuda:0")
    d = {k: torch.from_numpy(v).to(dev) for k, v in dict(cell=cell, pmax=pmax, psum=psum, pacc=pacc,
                                                          rs=row_slots).items()}
    olib = oracle.lib()
    for row in range(layers + 1):
        streams = rng.normal(size=(count, 4, dim)).astype(np.float32)
        olib.ndo_conf_pool_update(row, streams.ctypes.data, row_slots.ctypes.data, count, int(row == 0),
                                  probe_v.ctypes.data, probes, dim, pool_rows, want[0].ctypes.data,
                                  want[1].ctypes.data, want[2].ctypes.data, want[3].ctypes.data, None, None, None,
                                  None)
        ds = torch.from_numpy(streams).to(dev)
        _native.call("ndl_conf_pool_update", row, ds.data_ptr(), d["rs"].data_ptr(), count, int(row == 0),
                     probes_t.values, probes, dim, pool_rows, slots, d["cell"].data_ptr(), d["pmax"].data_ptr(),
                     d["psum"].data_ptr(), d["pacc"].data_ptr(), None, None, None, None, None)
    listed = np.array([3, 1, 4], np.int32)
    dl = torch.from_numpy(listed).to(dev)
    logits = torch.empty(listed.size, device=dev)
    _native.call("ndl_conf_logit", dl.data_ptr(), listed.size, d["psum"].data_ptr(), d["pacc"].data_ptr(), pool_rows,
                 dim, m.tensor("probe.gain", h).values, query_t.values, m.tensor("probe.row_bias", h).values, bias,
                 proj_t.values, queries, logits.data_ptr(), None, None)
    got = logits.cpu().numpy()
    for r, s in enumerate(listed):
        wp = np.zeros((queries, dim), np.float32)
        wl = olib.ndo_conf_logit(want[2][s].ctypes.data, want[3][s].ctypes.data, pool_rows, dim, gain.ctypes.data,
                                 qv.ctypes.data, rb.ctypes.data, bias, proj.ctypes.data, queries, wp.ctypes.data)
        assert np.float32(got[r]) == np.float32(wl), (r, got[r], wl)


def test_kronecker_mlp_runs_on_model_weights(loaded, oracle):
    """ndl_mlp_apply over several residual rows of a layer against the oracle's
    HadamardMlp restatement on the same (host) tensors, bit for bit (the
    condition softmax and the SiLU take the correctly rounded exponential on
    both sides)."""
    import torch

    from needle_cs_b200 import _native

    cact, a, m = loaded
    info = m.info
    dim, rows, cols = info["dim"], info["hada_rows"], info["hada_cols"]
    names = ["d1", "d2", "b2", "d3", "d4", "w1a", "w1b", "w2a", "w2b", "w3a", "w3b", "cond_v", "cond_u"]
    rng = np.random.default_rng(51)
    for layer in range(info["layers"]):
        host = [np.ascontiguousarray(m.host("layer.mlp." + n, layer)) for n in names]
        pre = m.host("layer.pre_hada", layer)
        pa, pb = m.host("hyper.perm_a"), m.host("hyper.perm_b")
        residual = rng.normal(size=(5, dim)).astype(np.float32)
        want = residual.copy()
        ptrs = (ctypes.c_void_p * 13)(*[h.ctypes.data for h in host])
        for t in range(5):
            oracle.lib().ndo_hadamard_mlp(ptrs, pre.ctypes.data, pa.ctypes.data, pb.ctypes.data, dim, rows, cols,
                                          0.5, want[t].ctypes.data)
        res = torch.from_numpy(residual).cuda()
        m.apply_mlp(layer, res, 0.5)
        got = res.cpu().numpy()
        delta = np.abs(want - residual).max()
        assert delta > 1e-3  # the MLP moves the rows
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), np.abs(got - want).max()
