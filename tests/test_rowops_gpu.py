"""Needle-3 row operations on the GPU (hyper-connection mixing, Sinkhorn,
conv taps, fake-A8 norms): the KernelTable slots 6-13 and 24 with host
pointers, and the batched device entry points, against the oracle's scalar
restatements (src/Needle/Scalar.cs:250-439, src/Needle/Ops.cs:800-812).

Bar: bit-exact, GateFakeA8 and Sinkhorn4x4 included (their MathF.Exp is the
correctly rounded exponential on both sides); Sinkhorn4x4's golden, a zero
matrix -> 0.25 everywhere, is exact.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

F = ctypes.c_float


def _p(a):
    return a.ctypes.data


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.fixture(scope="module")
def lib(pkg, cuda):
    return pkg.lib()


@pytest.fixture(scope="module")
def olib(oracle):
    return oracle.lib()


def _fill(oracle, seed, n, scale=2.0):
    return oracle.XorShift64(seed).fill_edges(n, scale)[:n].copy()


@pytest.mark.parametrize("dim", [1, 31, 384, 512])
def test_mix_combine_slots(lib, olib, oracle, dim):
    s = _fill(oracle, 11 + dim, 4 * dim)
    x, u, y = _fill(oracle, 12, dim), _fill(oracle, 13, dim), _fill(oracle, 14, dim)
    w = [0.3, -1.25, 0.875, 2.5]
    got, want = np.empty(dim, np.float32), np.empty(dim, np.float32)
    lib.ndl_kt_mix4(_p(s), dim, *w, _p(got))
    olib.ndo_mix4(_p(s), dim, *w, _p(want))
    assert np.array_equal(_bits(got), _bits(want))
    lib.ndl_kt_combine4(_p(s), dim, *w, _p(y), F(0.7), _p(got))
    olib.ndo_combine4(_p(s), dim, *w, _p(y), 0.7, _p(want))
    assert np.array_equal(_bits(got), _bits(want))
    lib.ndl_kt_combine_diff4(_p(s), dim, *w, _p(x), _p(u), F(1.5), _p(got))
    olib.ndo_combine_diff4(_p(s), dim, *w, _p(x), _p(u), 1.5, _p(want))
    assert np.array_equal(_bits(got), _bits(want))


def test_taps3_slot(lib, olib, oracle):
    width = 384
    taps = _fill(oracle, 21, 3 * width)
    buf = _fill(oracle, 22, 3 * width)  # x_{t-2}, x_{t-1}, x_t; current points at x_t
    cur = buf.ctypes.data + 2 * width * 4
    got, want = np.empty(width, np.float32), np.empty(width, np.float32)
    lib.ndl_kt_taps3(_p(taps), width, cur, _p(got))
    olib.ndo_taps3(_p(taps), width, ctypes.c_void_p(cur), _p(want))
    assert np.array_equal(_bits(got), _bits(want))


def test_sinkhorn_slot(lib, oracle, golden):
    out = np.empty(16, np.float32)
    lib.ndl_kt_sinkhorn4x4(_p(np.zeros(16, np.float32)), _p(out))
    assert np.array_equal(out, np.float32(golden["fixtures"]["Sinkhorn_zeros_4x4"]))
    rng = np.random.default_rng(3)
    for case in range(20):
        lg = (rng.normal(size=16) * (0.5 + case)).astype(np.float32)
        lib.ndl_kt_sinkhorn4x4(_p(lg), _p(out))
        want = oracle.sinkhorn4x4(lg)
        assert np.array_equal(out.view(np.uint32), want.view(np.uint32)), case


@pytest.mark.parametrize("n", [1, 5, 384, 512, 2048])
def test_fake_a8_slots(lib, olib, oracle, n):
    x = _fill(oracle, 31 + n, n, 3.0)
    scale = _fill(oracle, 32, n, 0.5)
    got = np.empty(n, np.float32)
    lib.ndl_kt_rms_fake_a8(_p(x), n, _p(got))
    assert np.array_equal(_bits(got), _bits(oracle.fake_a8_row(0, x)))
    lib.ndl_kt_centered_rms_fake_a8(_p(x), _p(scale), n, _p(got))
    assert np.array_equal(_bits(got), _bits(oracle.fake_a8_row(1, x, scale)))
    residual = _fill(oracle, 33, n)
    want = residual.copy()
    lib.ndl_kt_post_norm_add(_p(residual), _p(x), _p(scale), F(0.625), n)
    olib.ndo_post_norm_add(_p(want), _p(x), _p(scale), 0.625, n)
    assert np.array_equal(_bits(residual), _bits(want))
    gate = _fill(oracle, 34, n, 4.0)
    xg = x.copy()
    lib.ndl_kt_gate_fake_a8(_p(xg), _p(gate), n)
    want = oracle.fake_a8_row(2, x, gate)
    assert np.array_equal(_bits(xg), _bits(want))


def test_batched_device_entry_points(pkg, olib, oracle):
    import torch

    from needle_cs_b200 import _native

    dev = torch.device("cuda:0")
    n, dim = 257, 512
    rng = np.random.default_rng(9)
    s = rng.normal(size=(n, 4, dim)).astype(np.float32)
    w = rng.normal(size=(n, 4)).astype(np.float32)
    mix = rng.uniform(0, 1, (n, 16)).astype(np.float32)
    x, u = rng.normal(size=(n, dim)).astype(np.float32), rng.normal(size=(n, dim)).astype(np.float32)
    gates = rng.uniform(0, 2, (n, 4)).astype(np.float32)
    t = {k: torch.from_numpy(v).to(dev) for k, v in dict(s=s, w=w, mix=mix, x=x, u=u, g=gates).items()}
    out = torch.empty((n, dim), device=dev)
    _native.call("ndl_hc_mix4", t["s"].data_ptr(), dim, t["w"].data_ptr(), n, out.data_ptr(), None)
    nxt = torch.empty((n, 4, dim), device=dev)
    _native.call("ndl_hc_combine_diff4x4", t["s"].data_ptr(), dim, t["mix"].data_ptr(), t["x"].data_ptr(),
                 t["u"].data_ptr(), t["g"].data_ptr(), n, nxt.data_ptr(), None)
    logits = torch.from_numpy(rng.normal(size=(n, 16)).astype(np.float32) * 3).to(dev)
    sk = torch.empty((n, 16), device=dev)
    _native.call("ndl_hc_sinkhorn4x4", logits.data_ptr(), n, sk.data_ptr(), None)
    torch.cuda.synchronize()
    got_mix, got_next, got_sk = out.cpu().numpy(), nxt.cpu().numpy(), sk.cpu().numpy()
    lg = logits.cpu().numpy()
    want = np.empty(dim, np.float32)
    want4 = np.empty((4, dim), np.float32)
    for k in range(n):
        olib.ndo_mix4(_p(s[k]), dim, *[float(v) for v in w[k]], _p(want))
        assert np.array_equal(_bits(got_mix[k]), _bits(want)), k
        olib.ndo_combine_diff4x4(_p(s[k]), dim, _p(mix[k]), _p(x[k]), _p(u[k]), _p(gates[k]), _p(want4))
        assert np.array_equal(_bits(got_next[k]), _bits(want4)), k
        assert np.array_equal(_bits(got_sk[k]), _bits(oracle.sinkhorn4x4(lg[k]))), k

    # taps over chained triples, and the fake-A8 rows in every mode
    width, rows = 384, 64
    taps = torch.from_numpy(rng.normal(size=3 * width).astype(np.float32)).to(dev)
    triples = torch.from_numpy(rng.normal(size=(rows, 3, width)).astype(np.float32)).to(dev)
    tout = torch.empty((rows, width), device=dev)
    _native.call("ndl_taps3", taps.data_ptr(), width, triples.data_ptr(), rows, tout.data_ptr(), None)
    xr = torch.from_numpy(rng.normal(size=(rows, width)).astype(np.float32) * 3).to(dev)
    sc = torch.from_numpy(rng.uniform(-0.5, 0.5, width).astype(np.float32)).to(dev)
    fa = [torch.empty((rows, width), device=dev) for _ in range(2)]
    _native.call("ndl_fake_a8_rows", 0, xr.data_ptr(), None, None, rows, width, fa[0].data_ptr(), None)
    _native.call("ndl_fake_a8_rows", 1, xr.data_ptr(), sc.data_ptr(), None, rows, width, fa[1].data_ptr(), None)
    res = torch.from_numpy(rng.normal(size=(rows, width)).astype(np.float32)).to(dev)
    res0 = res.cpu().numpy()
    rg = torch.from_numpy(rng.uniform(0, 1, rows).astype(np.float32)).to(dev)
    _native.call("ndl_fake_a8_rows", 3, xr.data_ptr(), sc.data_ptr(), rg.data_ptr(), rows, width, res.data_ptr(), None)
    torch.cuda.synchronize()
    tp, tr, xh, sh = taps.cpu().numpy(), triples.cpu().numpy(), xr.cpu().numpy(), sc.cpu().numpy()
    gh, f0, f1, rh = rg.cpu().numpy(), fa[0].cpu().numpy(), fa[1].cpu().numpy(), res.cpu().numpy()
    got_t = tout.cpu().numpy()
    want = np.empty(width, np.float32)
    for r in range(rows):
        olib.ndo_taps3(_p(tp), width, ctypes.c_void_p(tr[r].ctypes.data + 2 * width * 4), _p(want))
        assert np.array_equal(_bits(got_t[r]), _bits(want)), r
        assert np.array_equal(_bits(f0[r]), _bits(oracle.fake_a8_row(0, xh[r]))), r
        assert np.array_equal(_bits(f1[r]), _bits(oracle.fake_a8_row(1, xh[r], sh))), r
        ref = res0[r].copy()
        olib.ndo_post_norm_add(_p(ref), _p(xh[r]), _p(sh), float(gh[r]), width)
        assert np.array_equal(_bits(rh[r]), _bits(ref)), r


@pytest.mark.parametrize("width", [384, 3072, 4100, 770])  # CTA-per-row kernel, then widths it does not take
def test_fake_a8_rows_batched(pkg, oracle, width):
    """ndl_fake_a8_rows modes 0 and 2 over many rows (mode 2: one gate row per
    row) equal the oracle's rows bit for bit."""
    import torch

    from needle_cs_b200 import _native

    dev = torch.device("cuda:0")
    rows = 19
    rng = np.random.default_rng(width)
    xh = (rng.normal(size=(rows, width)) * 3).astype(np.float32)
    gh = (rng.normal(size=(rows, width)) * 4).astype(np.float32)
    xr, gr = torch.from_numpy(xh).to(dev), torch.from_numpy(gh).to(dev)
    out = [torch.empty((rows, width), device=dev) for _ in range(2)]
    _native.call("ndl_fake_a8_rows", 0, xr.data_ptr(), None, None, rows, width, out[0].data_ptr(), None)
    _native.call("ndl_fake_a8_rows", 2, xr.data_ptr(), gr.data_ptr(), None, rows, width, out[1].data_ptr(), None)
    torch.cuda.synchronize()
    f0, f2 = out[0].cpu().numpy(), out[1].cpu().numpy()
    for r in range(rows):
        assert np.array_equal(_bits(f0[r]), _bits(oracle.fake_a8_row(0, xh[r]))), r
        assert np.array_equal(_bits(f2[r]), _bits(oracle.fake_a8_row(2, xh[r], gh[r]))), r


def test_float_helper_slots(lib, olib, oracle, golden):
    """Slots 14-21 and 23 against the oracle and the reference's goldens."""
    fx = golden["fixtures"]
    rng = np.random.default_rng(21)
    n = 777
    x = (rng.normal(size=n) * 2).astype(np.float32)
    b = (rng.normal(size=n)).astype(np.float32)
    got = np.empty(n, np.float32)
    lib.ndl_kt_rms_unit(_p(x), n, _p(got))
    inv = np.float32(olib.ndo_inverse_rms(_p(x), n))
    assert np.array_equal(_bits(got), _bits(x * inv))
    scale = (rng.uniform(-0.5, 0.5, n)).astype(np.float32)
    want = np.empty(n, np.float32)
    lib.ndl_kt_zero_centered_rms(_p(x), _p(scale), n, _p(got))
    olib.ndo_zero_centered_rms(_p(x), _p(scale), n, _p(want))
    assert np.array_equal(_bits(got), _bits(want))
    # Dot: sequential fp32 sum, and its golden
    d = lib.ndl_kt_dot(_p(x), _p(b), n)
    acc = np.float32(0)
    for i in range(n):
        acc = np.float32(acc + np.float32(x[i] * b[i]))
    assert np.float32(d).view(np.uint32) == acc.view(np.uint32)
    a8 = np.arange(1, 9, dtype=np.float32)
    assert lib.ndl_kt_dot(_p(a8), _p(a8[::-1].copy()), 8) == fx["Dot_1to8_8to1"]
    # AddScaled, ScaleAdd, MultiplyAccumulate: one rounding per operation
    dst = (rng.normal(size=n)).astype(np.float32)
    out = dst.copy()
    lib.ndl_kt_add_scaled(_p(out), _p(x), F(0.75), n)
    assert np.array_equal(_bits(out), _bits(dst + np.float32(0.75) * x))
    out = dst.copy()
    lib.ndl_kt_scale_add(_p(out), F(-1.5), _p(x), F(0.25), n)
    assert np.array_equal(_bits(out), _bits(np.float32(-1.5) * dst + np.float32(0.25) * x))
    out = dst.copy()
    lib.ndl_kt_multiply_accumulate(_p(out), _p(x), _p(b), n)
    assert np.array_equal(_bits(out), _bits(dst + x * b))
    # Softmax (exp: tolerance) and its goldens
    for inp, key in (([0, 0, 0], "Softmax_0_0_0"), ([1, 2, 3], "Softmax_1_2_3")):
        v = np.float32(inp)
        lib.ndl_kt_softmax(_p(v), 3)
        assert np.allclose(v, np.float32(fx[key]), rtol=2e-7, atol=1e-7)
    v, w = x.copy(), x.copy()
    lib.ndl_kt_softmax(_p(v), n)
    olib.ndo_softmax(_p(w), n)
    assert np.allclose(v, w, rtol=1e-6, atol=1e-12)
    # FakeA8: bit-exact, half-to-even ties at a unit scale
    v, w = x.copy(), x.copy()
    sc = lib.ndl_kt_fake_a8(_p(v), n)
    sw = olib.ndo_fake_a8(_p(w), n)
    assert np.float32(sc) == np.float32(sw) and np.array_equal(_bits(v), _bits(w))
    ties = np.float32([127.0, 0.5, 2.5, -0.5])
    lib.ndl_kt_fake_a8(_p(ties), 4)
    assert ties[1] == fx["FakeA8_tie_0_5"] and ties[2] == fx["FakeA8_tie_2_5"] and ties[3] == 0.0
    # Rope over 6 heads of 64 at position 37
    heads, hd = 6, 64
    cs, sn = oracle.rope_tables(10000.0, hd, 64)
    cs, sn = np.ascontiguousarray(cs.reshape(64, -1)[37]), np.ascontiguousarray(sn.reshape(64, -1)[37])
    q = (rng.normal(size=heads * hd)).astype(np.float32)
    r1, r2 = q.copy(), q.copy()
    lib.ndl_kt_rope(_p(r1), heads, hd, _p(cs), _p(sn))
    olib.ndo_rope(_p(r2), heads, hd, _p(cs), _p(sn))
    assert np.array_equal(_bits(r1), _bits(r2))
