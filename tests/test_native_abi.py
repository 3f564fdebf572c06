"""The C-ABI library loads on a CPU-only host and exports every declared symbol.

No compute call is made here; these checks need no GPU.
"""
import ctypes
import os
import re

import numpy as np

from conftest import ROOT


def declared_symbols():
    names = []
    for header in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if header.endswith(".h"):
            text = open(os.path.join(ROOT, "include", header)).read()
            names += re.findall(r"NDL_API\s+[^;(]*?\b(ndl_\w+)\s*\(", text)
    return names


def test_header_declares_symbols():
    names = declared_symbols()
    assert len(names) >= 10
    assert len(set(names)) == len(names)


def test_library_exports_every_declared_symbol(pkg):
    lib = ctypes.CDLL(pkg.LIB_PATH)
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol(pkg):
    import needle_cs_b200._native as native

    missing = [n for n in declared_symbols() if n not in native.SIGNATURES]
    assert not missing, missing


def test_status_strings(pkg):
    lib = pkg.lib()
    assert lib.ndl_status_string(0) == b"ok"
    assert lib.ndl_status_string(3) == b"ContextExhausted"
    assert lib.ndl_status_string(100) == b"invalid argument"
    assert b"sm_100a" in lib.ndl_version()


def test_f16_conversion_matches_ieee(pkg):
    lib = pkg.lib()
    rng = np.random.default_rng(1)
    vals = np.concatenate([rng.normal(size=2000) * 10.0 ** rng.integers(-9, 6, 2000),
                           [0.0, -0.0, 65504.0, 65520.0, 65519.99, 6.1e-5, 5.96e-8, 2.98e-8, 2.99e-8, 1e-9]])
    vals = vals.astype(np.float32)
    got = np.array([lib.ndl_f32_to_f16(float(v)) for v in vals], np.uint16)
    assert np.array_equal(got, vals.astype(np.float16).view(np.uint16))


def test_synth_host_is_deterministic(ops):
    a = ops.synth_normal_f32(1, 5, 30000)
    b = ops.synth_normal_f32(1, 5, 30000)
    assert np.array_equal(a, b)
    assert abs(a.mean()) < 0.03 and abs(a.std() - 1.0) < 0.03
    tail = ops.synth_normal_f32(1, 5, 100, first=29900)
    assert np.array_equal(tail, a[29900:])
    w = ops.synth_int8(0, 2, 100000)
    assert w.min() == -127 and w.max() == 127
    u = ops.synth_uniform_f16(0, 3, 10000, 0.001, 0.02).view(np.float16).astype(np.float32)
    assert u.min() >= 0.001 - 1e-6 and u.max() <= 0.02 + 1e-5


def test_device_count_without_gpu_is_an_error_not_a_crash(pkg):
    import torch

    n = ctypes.c_int(-1)
    st = pkg.lib().ndl_device_count(ctypes.byref(n))
    if torch.cuda.is_available():
        assert st == 0 and n.value >= 1
    else:
        assert st in (0, 106) and n.value == 0
