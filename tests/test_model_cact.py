"""The .cact loader on the host (no GPU): ndl_model_load with device -1.

Archives are written by tests/cact_support.py in the reference's layout.  The
cases follow the reference's own format tests
(tests/Needle.Tests/FormatTests.cs:155-248, LoadingTests.cs:128-145): short
and empty input, wrong and zero magic, truncation, unsupported head,
convolution and Engram geometry, each with the facts and the guidance
sentence in the message.  Added here:
 * the loader's own checks (a record of the wrong kind, no tokenizer, a walk
   past the table, a permutation entry out of range, a short codebook);
 * the fp16 rule over all 65,536 patterns, exact and upstream
   (MatMulTests.cs:88-113 checks the exact decode the same way);
 * the codebooks against the oracle's Codebook.Fill.
"""
import numpy as np
import pytest

from cact_support import CQ, FP32, GEOMETRY, Archive, half_to_single

GUIDANCE = "CONTRIBUTING.md, section \"Refreshing the upstream model\""


@pytest.fixture(scope="module")
def cact(pkg):
    import importlib

    return importlib.import_module("needle_cs_b200.model")


def _check_entries(model, archive, cact):
    names = model.tensors()
    want = [(r[0], r[1]) for r in archive.records if r[0] != "tokenizer"]
    assert names == want
    for role, index, dtype, shape, payload, bits, exp in archive.records:
        if role == "tokenizer":
            assert model.tokenizer_blob() == payload
            continue
        t = model.tensor(role, index)
        assert (t.dtype, t.ndim, list(t.shape)[:t.ndim]) == (dtype, len(shape), list(shape))
        assert t.values is None and t.indices is None  # host only
        if exp[0] == "cq":
            _, codes, norms, rows, cols, b = exp
            assert (t.kind in (cact.CQ, cact.CQ_ROWS), t.rows, t.cols, t.bits) == (True, rows, cols, b)
            assert t.bytes == codes.nbytes + norms.nbytes
        elif exp[0] == "perm":
            assert t.kind == cact.PERMUTATION
            assert np.array_equal(model.host(role, index), exp[1])
        else:
            assert t.kind == cact.DENSE
            got = model.host(role, index)
            want_v = half_to_single(exp[1], not model.info["has_audio"]) if exp[0] == "dense16" else exp[1]
            assert np.array_equal(got.view(np.uint32), want_v.view(np.uint32)), (role, index)


def test_synthetic_archive_loads_with_every_role(cact):
    a = Archive(seed=1).standard(probe_codes=(2, 1))
    with cact.Model.from_bytes(a.build()) as m:
        info = m.info
        for k in ("vocab", "dim", "heads", "kv_heads", "layers", "qk_dim", "v_dim", "hada_n", "engram_slots",
                  "engram_tables", "engram_dilation", "kv_window", "sliding_window", "global_mask"):
            assert info[k] == GEOMETRY[k], k
        assert info["orders"] == GEOMETRY["orders"] and info["sites"] == GEOMETRY["sites"]
        assert info["rope_theta"] == GEOMETRY["rope_theta"]
        assert (info["hada_rows"], info["hada_cols"]) == (8, 16)
        assert info["magic"] == 0x05E12A84 and info["tensors"] == len(a.records)
        assert info["probe_codes"] == [2, 1]
        assert (info["confidence_head"], info["embedding_head"]) == (0, 1)
        assert info["has_confidence"] and info["has_embedding_head"] and not info["has_audio"]
        assert info["device"] == -1 and info["tokenizer_bytes"] == len(a.records[-1][4])
        _check_entries(m, a, cact)
        assert m.tensor("probe.probe_vectors", 1).kind == cact.CQ_ROWS
        assert m.tensor("layer.q", 1).kind == cact.CQ


def test_archives_without_heads_with_a_router_and_with_audio(cact):
    for kwargs in (dict(probe_codes=()), dict(probe_codes=(3, 2)), dict(audio=True)):
        a = Archive(seed=2).standard(**kwargs)
        with cact.Model.from_bytes(a.build()) as m:
            _check_entries(m, a, cact)
            assert m.info["has_audio"] == bool(kwargs.get("audio"))
            assert m.info["probe_heads"] == len(kwargs.get("probe_codes", ()))


@pytest.mark.parametrize("audio", [False, True])
def test_half_rule_on_all_patterns(cact, audio):
    """Without audio weights every fp16 record decodes exactly
    (HalfToSingle); with them, records before the audio section decode by
    HalfToSingleUpstream (subnormals read as normals)."""
    patterns = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    a = Archive(seed=3).standard(audio=audio, final_norm=patterns)
    with cact.Model.from_bytes(a.build()) as m:
        got = m.host("final_norm")
    want = half_to_single(patterns, exact=not audio)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert got[0x8000] == 0 and not np.signbit(got[0x8000])  # -0 reads as +0
    assert got[0x7C00] == 65536.0  # exponent 31 is an ordinary exponent
    assert (got[1] == np.float32(2.0 ** -24)) == (not audio)


def test_codebooks_equal_codebook_fill(cact, oracle):
    a = Archive(seed=4).standard()
    with cact.Model.from_bytes(a.build()) as m:
        for role, count, lo in (("layer.q", 4, 0), ("embedding", 16, 12)):
            book = m.tensor(role, 0).book.contents
            want = oracle.codebook(a.levels[lo:lo + count], count)
            assert bytes(book.bytes) == bytes(want.bytes)
            assert np.array_equal(np.array(book.levels, np.float32), np.array(want.levels, np.float32))
            assert np.float32(book.byte_scale) == np.float32(want.byte_scale)


# -- the reference's format tests ------------------------------------------------


def test_short_and_empty_inputs_name_the_header_size(cact):
    for data in (b"", bytes(100)):
        with pytest.raises(cact.InvalidDataError) as e:
            cact.Model.from_bytes(data)
        assert f"the file has {len(data)} bytes" in str(e.value)
        assert "196-byte header" in str(e.value) and GUIDANCE in str(e.value)


def test_wrong_and_zero_magic(cact):
    data = bytearray(4096)
    data[:4] = (0xDEADBEEF).to_bytes(4, "little")
    with pytest.raises(cact.InvalidDataError) as e:
        cact.Model.from_bytes(bytes(data))
    assert "found magic 0xDEADBEEF" in str(e.value) and "0x05E12A84" in str(e.value)
    assert GUIDANCE in str(e.value)
    with pytest.raises(cact.InvalidDataError) as e:
        cact.Model.from_bytes(bytes(4096))
    assert "found magic 0x00000000" in str(e.value)


def test_truncated_archive_names_the_lengths(cact):
    whole = Archive(seed=5).standard().build()
    for keep in (300, 1000, len(whole) // 2, len(whole) - 1):
        with pytest.raises(cact.InvalidDataError) as e:
            cact.Model.from_bytes(whole[:keep])
        assert "truncated" in str(e.value) and f"the file has {keep} bytes" in str(e.value)
        assert GUIDANCE in str(e.value)


def _patched(word, value):
    a = Archive(seed=6).standard()
    h = a.header_words()
    h[word] = value
    return a.build(header=h)


def test_unsupported_geometry_names_found_and_supported(cact):
    with pytest.raises(cact.NotSupportedError) as e:
        cact.Model.from_bytes(_patched(11, 32))
    assert "unsupported head geometry" in str(e.value) and "QkDim=32" in str(e.value) and "QkDim=48" in str(e.value)
    assert GUIDANCE in str(e.value)
    with pytest.raises(cact.NotSupportedError) as e:
        cact.Model.from_bytes(_patched(19, 5))
    assert "ConvTaps=5" in str(e.value) and "ConvTaps=3" in str(e.value)
    with pytest.raises(cact.NotSupportedError) as e:
        cact.Model.from_bytes(_patched(26, 9))
    assert "found 9 orders" in str(e.value) and "at most 4 orders" in str(e.value)
    with pytest.raises(cact.NotSupportedError) as e:
        cact.Model.from_bytes(_patched(14, 100))  # 100 = 16 x 6.25: no rows x columns split
    assert "unsupported MLP geometry" in str(e.value) and "HadaN=100" in str(e.value)


# -- checks of this loader ----------------------------------------------------------


def _replace(archive, role, index, record):
    i = next(k for k, r in enumerate(archive.records) if r[0] == role and r[1] == index)
    archive.records[i] = record


def test_a_record_of_the_wrong_kind_is_malformed(cact):
    a = Archive(seed=7).standard()
    _replace(a, "layer.k", 1, ("layer.k", 1, FP32, [16], bytes(64), 0, None))
    with pytest.raises(cact.InvalidDataError, match="2- or 4-bit CQ tensor expected"):
        cact.Model.from_bytes(a.build())
    a = Archive(seed=7).standard()
    _replace(a, "final_norm", 0, ("final_norm", 0, CQ, [1, 128], bytes(68), 2, None))
    with pytest.raises(cact.InvalidDataError, match="dense tensor expected"):
        cact.Model.from_bytes(a.build())
    a = Archive(seed=7).standard()
    _replace(a, "layer.v", 0, ("layer.v", 0, CQ, [4, 100], bytes(200), 2, None))
    with pytest.raises(cact.InvalidDataError, match="CQ group of 128 expected"):
        cact.Model.from_bytes(a.build())


def test_missing_tokenizer_and_short_tables(cact):
    a = Archive(seed=8).standard()
    a.records.pop()  # no tokenizer: the last record is a probe tensor
    with pytest.raises(cact.InvalidDataError, match="tokenizer blob missing"):
        cact.Model.from_bytes(a.build())
    a = Archive(seed=8).standard()
    del a.records[10:]
    with pytest.raises(cact.InvalidDataError, match="tensor table ends after 10 records"):
        cact.Model.from_bytes(a.build())


def test_permutation_and_codebook_checks(cact):
    a = Archive(seed=9).standard()
    bad = np.arange(128, dtype=np.float32)
    bad[5] = 128
    _replace(a, "hyper.perm_b", 0, ("hyper.perm_b", 0, FP32, [128], bad.tobytes(), 0, None))
    with pytest.raises(cact.InvalidDataError, match=r"permutation entry 5 .* is 128, outside \[0, 128\)"):
        cact.Model.from_bytes(a.build())
    a = Archive(seed=9).standard()
    a.levels = a.levels[:20]
    with pytest.raises(cact.InvalidDataError, match="codebook holds 20 levels"):
        cact.Model.from_bytes(a.build())


def test_cq_larger_than_its_bytes_is_malformed(cact):
    a = Archive(seed=10).standard()
    _replace(a, "site.key", 0, ("site.key", 0, CQ, [128, 128], bytes(1000), 2, None))
    with pytest.raises(cact.InvalidDataError, match="codes and norms need"):
        cact.Model.from_bytes(a.build())


def test_missing_file_raises_file_not_found(cact, tmp_path):
    with pytest.raises(FileNotFoundError):
        cact.Model.open(str(tmp_path / "absent.cact"))


def test_upload_to_a_missing_device_is_an_error(cact):
    """A device index no GPU answers to fails with NDL_ERR_NO_DEVICE and no model."""
    a = Archive(seed=11).standard()
    with pytest.raises(cact.NeedleError) as e:
        cact.Model.from_bytes(a.build(), device=4096)
    assert e.value.status == 106 and "no CUDA device 4096" in str(e.value)
