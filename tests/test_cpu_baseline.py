"""The AVX2 CPU baseline (oracle/avx2_decoder.c) and the oracle's own copy
of the synthetic generator, on the CPU.

* The baseline's int8 linear (Gemv.Block's maddubs/madd group dots, the
  group fold by fused multiply-adds) returns the scalar oracle's y bit for
  bit at cfg1's shapes (M = 1 and 16 tokens of [2048, 512]) and at a row
  count that is not a multiple of its 8-row blocks.
* Its batched decode step returns, for every row, the logits the scalar
  oracle's decoder row gives, bit for bit, and writes the same K/V.
* The oracle's generator and decoder tensors equal the CUDA library's host
  generators', so the CPU arm needs nothing from the library.
"""
import numpy as np
import pytest


@pytest.mark.parametrize("m,n", [(1, 2048), (16, 2048), (5, 1000)])
def test_avx2_linear_equals_scalar_oracle(oracle, m, n):
    k = 512
    x = oracle.synth_normal(0, 1, m * k).reshape(m, k)
    w = oracle.synth_int8(0, 2, n * k).reshape(n, k)
    sw = oracle.synth_uniform_f16(0, 3, n * (k // 32), 0.001, 0.02).reshape(n, k // 32)
    q, sa = oracle.quantize_rows(x)
    ref = oracle.matmul_i8g32(q, sa, w, sw)
    got = oracle.matmul_i8g32_avx2(q, sa, w, sw, threads=4)
    assert np.array_equal(got, ref)


def test_avx2_decode_step_equals_scalar_rows(oracle):
    cfg = oracle.DecoderConfig(layers=2, dim=128, heads=2, head_dim=64, ffn=256, vocab=1000, seed=7)
    dec = oracle.synthetic_decoder(cfg, 320)
    avx = oracle.AVX2Decoder(dec)
    lengths = [1, 5, 64, 65, 130, 257]
    tokens = [3, 999, 0, 17, 500, 42]
    kv_a = [dec.new_kv() for _ in lengths]
    kv_b = [dec.new_kv() for _ in lengths]
    for r, n in enumerate(lengths):
        oracle.synthetic_prefix_kv(dec, kv_a[r], n, 3, 50 + r)
        oracle.synthetic_prefix_kv(dec, kv_b[r], n, 3, 50 + r)
    for step in range(2):
        pos = [n + step for n in lengths]
        got = avx.step(tokens, pos, kv_a, threads=3)
        for r in range(len(lengths)):
            ref = dec.row(tokens[r], pos[r], kv_b[r])
            assert np.array_equal(got[r], ref), (step, r)
        for key in ("k", "v", "ks", "vs"):
            for r in range(len(lengths)):
                assert np.array_equal(kv_a[r][key], kv_b[r][key]), (step, r, key)
        tokens = [int(np.argmax(got[r])) for r in range(len(lengths))]
    avx.close()


def test_oracle_generator_equals_library_host_generator(pkg, ops, oracle):
    for seed, stream, first in ((1, 100, 0), (5, 3, 12345), (3, 1 << 40, 7)):
        assert np.array_equal(oracle.synth_int8(seed, stream, 4096, first=first),
                              ops.synth_int8(seed, stream, 4096, first=first))
        assert np.array_equal(oracle.synth_uniform_f16(seed, stream, 4096, 0.001, 0.02, first=first),
                              ops.synth_uniform_f16(seed, stream, 4096, 0.001, 0.02, first=first))
        assert np.array_equal(oracle.synth_normal_f16(seed, stream, 4096, 0.02, first=first),
                              ops.synth_normal_f16(seed, stream, 4096, 0.02, first=first))
        assert np.array_equal(oracle.synth_normal(seed, stream, 4096, first=first),
                              ops.synth_normal_f32(seed, stream, 4096, first=first))


def test_oracle_decoder_tensors_equal_the_library_host_build(pkg, oracle):
    import importlib

    syn = importlib.import_module("needle_cs_b200.synthetic")
    eng_mod = importlib.import_module("needle_cs_b200.engine")
    model = eng_mod.SyntheticDecoder(layers=2, dim=128, heads=2, head_dim=64, ffn=256, vocab=1000, seed=7)
    layers, fnorm, emb, wh, sh = syn.decoder_weights(model)
    cfg = oracle.DecoderConfig(layers=2, dim=128, heads=2, head_dim=64, ffn=256, vocab=1000, seed=7)
    dec = oracle.synthetic_decoder(cfg, 64)
    keep = dec._keep
    for l in range(2):
        for name, arr in layers[l].items():
            assert any(a is not None and a.dtype == arr.dtype and a.shape == arr.shape and np.array_equal(a, arr)
                       for a in keep if isinstance(a, np.ndarray)), (l, name)
    for arr in (fnorm, emb, wh, sh):
        assert any(isinstance(a, np.ndarray) and a.shape == arr.shape and np.array_equal(a, arr) for a in keep)
