"""ctypes wrapper of the CPU parity oracle (oracle/build/liboracle.so).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and
the CPU-baseline legs of bench.py as the checker; never by the library.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "build", "liboracle.so")

_c = ctypes
P = _c.c_void_p
I = _c.c_int
F = _c.c_float
U64 = _c.c_uint64
PU64 = _c.POINTER(_c.c_uint64)

_SIGS = {
    "ndo_xorshift_next": (U64, [PU64]),
    # the Whistle front end (whistle_oracle.c)
    "ndo_log_rn": (F, [F]),
    "ndo_log_rn_array": (None, [P, I, P]),
    "ndo_frontend_tables": (None, [I, I, P, I, P, P, P, P, P, P]),
    "ndo_mel_frame": (F, [P, I, I, P, P, P, P, P, I, P, P, P]),
    "ndo_normalize_columns": (None, [P, I, I]),
    "ndo_whistle_rope_tables": (None, [F, I, I, P, P]),
    "ndo_cross_position_tables": (None, [I, I, P, P]),
    "ndo_silu": (None, [P, I]),
    "ndo_glu": (None, [P, P, P, I]),
    "ndo_multiply_by_sigmoid": (None, [P, P, I]),
    "ndo_xorshift_int": (I, [PU64, I, I]),
    "ndo_xorshift_float": (F, [PU64, F]),
    "ndo_fill_uniform": (None, [P, I, PU64, F]),
    "ndo_fill_edges": (None, [P, I, PU64, F]),
    "ndo_fill_sbyte": (None, [P, I, PU64, I]),
    "ndo_fill_bytes": (None, [P, I, PU64, I]),
    "ndo_half_bits": (_c.c_uint16, [F]),
    "ndo_abs_max": (F, [P, I]),
    "ndo_quantize_int8": (F, [P, I, P]),
    "ndo_quantize_rows": (None, [P, I, I, P, P]),
    "ndo_fake_a8": (F, [P, I]),
    "ndo_half_to_single": (F, [_c.c_uint16]),
    "ndo_exp_rn": (None, [P, I, P]),
    "ndo_exp_simd": (None, [P, I, P]),
    "ndo_hadamard128": (None, [P, P]),
    "ndo_planes": (None, [P, I, P, _c.POINTER(I)]),
    "ndo_sigmoid": (F, [F]),
    "ndo_softmax": (None, [P, I]),
    "ndo_rope": (None, [P, I, I, P, P]),
    "ndo_rope_tables": (None, [F, I, I, P, P]),
    "ndo_inverse_rms": (F, [P, I]),
    "ndo_rms_norm": (None, [P, P, I, P]),
    "ndo_zero_centered_rms": (None, [P, P, I, P]),
    "ndo_swiglu": (None, [P, P, I, P]),
    "ndo_codebook_fill": (None, [P, P, I]),
    "ndo_prepare_cq": (None, [P, I, I, I, P, P, P, I]),
    "ndo_matmul_rows_cq": (None, [P, P, P, I, I, I, P, P, P, I, I, P, I, I, I]),
    "ndo_gather_row_cq": (None, [P, P, P, I, I, I, P]),
    "ndo_mix4": (None, [P, I, F, F, F, F, P]),
    "ndo_combine4": (None, [P, I, F, F, F, F, P, F, P]),
    "ndo_combine_diff4": (None, [P, I, F, F, F, F, P, P, F, P]),
    "ndo_combine_diff4x4": (None, [P, I, P, P, P, P, P]),
    "ndo_taps3": (None, [P, I, P, P]),
    "ndo_sinkhorn4x4": (None, [P, P]),
    "ndo_rms_fake_a8": (None, [P, I, P]),
    "ndo_centered_rms_fake_a8": (None, [P, P, I, P]),
    "ndo_gate_fake_a8": (None, [P, P, I]),
    "ndo_post_norm_add": (None, [P, P, P, F, I]),
    "ndo_hadamard_mlp": (None, [P, P, P, P, I, I, I, F, P]),
    "ndo_engram_hash": (None, [P, P, I, P, P, P, I, I, I, P]),
    "ndo_engram_conv": (None, [P, P, P, I, P, I, I, P, P]),
    "ndo_engram_gate": (None, [P, P, P, I, P]),
    "ndo_conf_pool_update": (None, [I, P, P, I, I, P, I, I, I, P, P, P, P, P, P, P, P]),
    "ndo_conf_logit": (F, [P, P, I, I, P, P, P, F, P, I, P]),
    "ndo_matmul_i8g32": (None, [P, P, I, I, P, P, I, P, P, I]),
    "ndo_attention_head": (None, [P, F, P, P, P, P, I, I, I, I, I, I, I, F, P, P, P]),
    "ndo_attention_head_simd": (None, [P, F, P, P, P, P, I, I, I, I, I, I, I, F, P, P]),
    "ndo_merge_partials": (None, [P, I, I, I, I, P]),
    "ndo_argmax": (I, [P, I]),
    "ndo_argmax_masked": (I, [P, P, I, I]),
    "ndo_best_probability": (F, [P, I, F]),
    "ndo_argmax_sparse": (I, [P, P, I, _c.POINTER(F)]),
    "ndo_argmax_masked_with_probability": (I, [P, P, I, I, P, _c.POINTER(F)]),
    "ndo_topk_logsoftmax": (None, [P, I, I, P, P, P, I]),
    "ndo_decoder_row": (I, [P, I, I, I, P, P, P, P, P, P, P]),
    "ndo_decoder_row_cross": (I, [P, I, I, I, P, P, P, P, P, P, I, P, P, P, P, P]),
    "ndo_cross_memory": (I, [P, I, P, I, P, P, P, P]),
    "ndo_synth_normal": (None, [U64, U64, U64, _c.c_size_t, F, P]),
    "ndo_synth_uniform": (None, [U64, U64, U64, _c.c_size_t, F, F, P]),
    "ndo_synth_int8": (None, [U64, U64, U64, _c.c_size_t, P]),
    "ndb_model_create": (P, [P]),
    "ndb_model_destroy": (None, [P]),
    "ndb_decode_step": (I, [P, I, P, P, I, P, P, P, P, P, P, P, I]),
    "ndb_matmul_i8g32": (None, [P, P, I, I, P, P, I, P, I, I]),
    "ndb_linear_create": (P, [P, P, I, I]),
    "ndb_linear_run": (None, [P, P, P, I, P, I, I]),
    "ndb_linear_destroy": (None, [P]),
}

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"oracle not built: {LIB_PATH} (run make -C oracle)")
        h = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _lib = h
    return _lib


def ptr(a):
    return None if a is None else a.ctypes.data


class XorShift64:
    """Port of the reference test RNG (Conformance.cs:10-38), state in C."""

    def __init__(self, seed):
        self.state = _c.c_uint64(seed if seed != 0 else 0x9E3779B97F4A7C15)

    def next(self):
        return lib().ndo_xorshift_next(_c.byref(self.state))

    def next_int(self, lo, hi):
        return lib().ndo_xorshift_int(_c.byref(self.state), lo, hi)

    def next_float(self, scale):
        return lib().ndo_xorshift_float(_c.byref(self.state), scale)

    def fill_edges(self, n, scale):
        x = np.empty(max(n, 1), np.float32)
        lib().ndo_fill_edges(ptr(x), max(n, 1), _c.byref(self.state), scale)
        return x

    def fill_uniform(self, n, scale):
        x = np.empty(max(n, 1), np.float32)
        lib().ndo_fill_uniform(ptr(x), max(n, 1), _c.byref(self.state), scale)
        return x

    def fill_sbyte(self, n, extremes):
        x = np.empty(max(n, 1), np.int8)
        lib().ndo_fill_sbyte(ptr(x), max(n, 1), _c.byref(self.state), int(extremes))
        return x

    def fill_bytes(self, n, extremes):
        x = np.empty(max(n, 1), np.uint8)
        lib().ndo_fill_bytes(ptr(x), max(n, 1), _c.byref(self.state), int(extremes))
        return x


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def exp_rn(x):
    """MathF.Exp as the oracle computes it (float in, float out)."""
    x = f32(x)
    y = np.empty_like(x)
    lib().ndo_exp_rn(ptr(x), x.size, ptr(y))
    return y


def exp_simd(x):
    """Ops.Exp, the reference's SIMD exponential, as the oracle restates it."""
    x = f32(x)
    y = np.empty_like(x)
    lib().ndo_exp_simd(ptr(x), x.size, ptr(y))
    return y


def quantize_int8(x):
    x = f32(x)
    q = np.empty(x.size, np.int8)
    s = lib().ndo_quantize_int8(ptr(x), x.size, ptr(q))
    return q, s


def quantize_rows(x):
    x = f32(x)
    rows, cols = x.shape
    q = np.empty((rows, cols), np.int8)
    s = np.empty(rows, np.float32)
    lib().ndo_quantize_rows(ptr(x), rows, cols, ptr(q), ptr(s))
    return q, s


def matmul_i8g32(q, sa, w, sw, want_acc=False):
    q = np.ascontiguousarray(q, np.int8)
    sa = f32(sa)
    w = np.ascontiguousarray(w, np.int8)
    sw = np.ascontiguousarray(sw, np.uint16)
    m, k = q.shape
    n = w.shape[0]
    y = np.empty((m, n), np.float32)
    acc = np.empty((m, n, k // 32), np.int32) if want_acc else None
    lib().ndo_matmul_i8g32(ptr(w), ptr(sw), n, k, ptr(q), ptr(sa), m, ptr(acc), ptr(y), n)
    return (y, acc) if want_acc else y


class Codebook(_c.Structure):
    """Codebook (src/Needle/Model.cs:36-52): levels, level bytes, byte scale."""
    _fields_ = [("levels", _c.c_float * 16), ("bytes", _c.c_uint8 * 32), ("byte_scale", _c.c_float)]


def codebook(levels, count):
    """Codebook.Fill over the first `count` levels."""
    book = Codebook()
    lv = f32(np.resize(np.asarray(levels, np.float32), 16))
    lib().ndo_codebook_fill(_c.byref(book), ptr(lv), count)
    return book


def prepare_cq(x, bits):
    """Quant.PrepareRange scalar branch: (values [tokens][cols], scales and
    offsets [tokens][stride], stride) for x [tokens][cols]."""
    x = f32(x)
    tokens, cols = x.shape
    groups = cols // 128
    stride = (groups + 7) & ~7
    vals = np.zeros((tokens, cols), np.int8)
    sc = np.zeros((tokens, stride), np.float32)
    off = np.zeros((tokens, stride), np.float32)
    lib().ndo_prepare_cq(ptr(x), tokens, cols, bits, ptr(vals), ptr(sc), ptr(off), stride)
    return vals, sc, off, stride


def matmul_rows_cq(indices, norms, book, bits, vals, sc, off, row_start=0, row_end=None, y=None):
    """Scalar.MatMulRows on CQ weights: y [tokens][rows], rows outside
    [row_start, row_end) left as given."""
    indices = np.ascontiguousarray(indices, np.uint8)
    norms = np.ascontiguousarray(norms, np.uint16)
    tokens, cols = vals.shape
    rows = norms.size // (cols // 128)
    row_end = rows if row_end is None else row_end
    y = np.zeros((tokens, rows), np.float32) if y is None else y
    lib().ndo_matmul_rows_cq(ptr(indices), ptr(norms), _c.byref(book), rows, cols, bits, ptr(vals), ptr(sc),
                             ptr(off), sc.shape[1], tokens, ptr(y), y.shape[1], row_start, row_end)
    return y


def gather_row_cq(indices, norms, levels, bits, row):
    """Quant.GatherRow: CQ row `row` decoded and rotated back per group."""
    indices = np.ascontiguousarray(indices, np.uint8)
    norms = np.ascontiguousarray(norms, np.uint16)
    cols = indices.shape[1] * 8 // bits
    out = np.empty(cols, np.float32)
    lib().ndo_gather_row_cq(ptr(indices), ptr(norms), ptr(f32(np.resize(np.asarray(levels, np.float32), 16))), cols,
                            bits, row, ptr(out))
    return out


def sinkhorn4x4(logits):
    """Scalar.Sinkhorn4x4 on one 4x4 logit matrix."""
    lg = f32(np.asarray(logits, np.float32).reshape(16))
    out = np.empty(16, np.float32)
    lib().ndo_sinkhorn4x4(ptr(lg), ptr(out))
    return out


def fake_a8_row(mode, x, aux=None):
    """RmsFakeA8 (mode 0), CenteredRmsFakeA8 (1, aux = scale), GateFakeA8 (2,
    aux = gate) on one row."""
    x = f32(x).copy()
    out = np.empty_like(x)
    if mode == 0:
        lib().ndo_rms_fake_a8(ptr(x), x.size, ptr(out))
    elif mode == 1:
        lib().ndo_centered_rms_fake_a8(ptr(x), ptr(f32(aux)), x.size, ptr(out))
    else:
        lib().ndo_gate_fake_a8(ptr(x), ptr(f32(aux)), x.size)
        out = x
    return out


def rms_norm(x, w):
    x = f32(x)
    w = f32(w)
    out = np.empty_like(x)
    for r in range(x.shape[0]):
        lib().ndo_rms_norm(ptr(x[r]), ptr(w), x.shape[1], ptr(out[r]))
    return out


def softmax(s):
    s = f32(s).copy()
    lib().ndo_softmax(ptr(s), s.size)
    return s


def argmax_masked(x, mask, length):
    x = f32(x)
    mask = np.ascontiguousarray(mask, np.uint32)
    return lib().ndo_argmax_masked(ptr(x), ptr(mask), mask.size, length)


def best_probability(values, best):
    values = f32(values)
    return lib().ndo_best_probability(ptr(values), values.size, best)


def argmax_sparse(values, ids):
    """ArgMaxSparse over a sparse head list: (picked id or -1, probability)."""
    values = f32(values)
    ids = np.ascontiguousarray(ids, np.int32)
    assert values.size == ids.size
    p = _c.c_float()
    best = lib().ndo_argmax_sparse(ptr(values), ptr(ids), values.size, _c.byref(p))
    return best, p.value


def argmax_masked_with_probability(x, mask, length):
    x = f32(x)
    mask = np.ascontiguousarray(mask, np.uint32)
    scratch = np.empty(max(x.size, 1), np.float32)
    p = _c.c_float()
    best = lib().ndo_argmax_masked_with_probability(ptr(x), ptr(mask), mask.size, length, ptr(scratch),
                                                    _c.byref(p))
    return best, p.value


def topk_logsoftmax(x, k, mask_special_023=False, want_probs=True):
    x = f32(x)
    idx = np.empty(k, np.int32)
    lp = np.empty(k, np.float32)
    pr = np.empty(k, np.float32) if want_probs else None
    lib().ndo_topk_logsoftmax(ptr(x), x.size, k, ptr(idx), ptr(lp), ptr(pr), int(mask_special_023))
    return idx, lp, pr


def attention_head(query, query_scale, keys, key_scales, values, value_scales, key_stride, value_stride,
                   scale_stride, first, last, qk_dim, v_dim, inv_sqrt_dim, probabilities=None):
    count = last - first + 1
    scores = np.empty(max(count, 1) + 8, np.float32)
    out = np.empty(v_dim, np.float32)
    lib().ndo_attention_head(ptr(query), query_scale, ptr(keys), ptr(key_scales), ptr(values), ptr(value_scales),
                             key_stride, value_stride, scale_stride, first, last, qk_dim, v_dim, inv_sqrt_dim,
                             ptr(scores), ptr(out), ptr(probabilities))
    return out


def attention_head_simd(query, query_scale, keys, key_scales, values, value_scales, key_stride, value_stride,
                        scale_stride, first, last, qk_dim, v_dim, inv_sqrt_dim):
    """Attention.GroupAvx2 on one head of an unsplit tile (the AVX2 tier)."""
    count = last - first + 1
    scores = np.empty(max(count, 1) + 8, np.float32)
    out = np.empty(v_dim, np.float32)
    lib().ndo_attention_head_simd(ptr(query), query_scale, ptr(keys), ptr(key_scales), ptr(values),
                                  ptr(value_scales), key_stride, value_stride, scale_stride, first, last, qk_dim,
                                  v_dim, inv_sqrt_dim, ptr(scores), ptr(out))
    return out


def merge_partials(partials, count, heads, stride, peak_off):
    partials = f32(partials)
    out = np.empty(heads * 64, np.float32)
    lib().ndo_merge_partials(ptr(partials), count, heads, stride, peak_off, ptr(out))
    return out


def rope_tables(theta, qk_dim, positions):
    half = qk_dim // 2
    c = np.empty((positions, half), np.float32)
    s = np.empty((positions, half), np.float32)
    lib().ndo_rope_tables(theta, qk_dim, positions, ptr(c), ptr(s))
    return c, s


class _Decoder(_c.Structure):
    _fields_ = [("layers", I), ("dim", I), ("heads", I), ("head_dim", I), ("ffn", I), ("vocab", I),
                ("rope_theta", F), ("eps", F)] + [
        (name, _c.POINTER(P)) for name in ("w_qkv", "s_qkv", "w_o", "s_o", "w_gu", "s_gu", "w_d", "s_d",
                                           "attn_norm", "ffn_norm")] + [
        ("final_norm", P), ("embedding", P), ("w_head", P), ("s_head", P)] + [
        (name, _c.POINTER(P)) for name in ("w_cq", "s_cq", "w_ckv", "s_ckv", "w_co", "s_co", "cross_norm")]


LAYER_TENSORS = {"w_qkv": np.int8, "s_qkv": np.uint16, "w_o": np.int8, "s_o": np.uint16, "w_gu": np.int8,
                 "s_gu": np.uint16, "w_d": np.int8, "s_d": np.uint16, "attn_norm": np.float32,
                 "ffn_norm": np.float32}
# per-layer tensors of the cross-attention blocks (Whistle-shaped decoder)
CROSS_TENSORS = {"w_cq": np.int8, "s_cq": np.uint16, "w_ckv": np.int8, "s_ckv": np.uint16, "w_co": np.int8,
                 "s_co": np.uint16, "cross_norm": np.float32}


class Decoder:
    """The synthetic decoder on the CPU (ndo_decoder_row), fed with weights
    copied from the engine under test."""

    def __init__(self, cfg, layer_weights, final_norm, embedding, w_head, s_head, capacity):
        """layer_weights[l] holds LAYER_TENSORS and, for a decoder with
        cross-attention, CROSS_TENSORS."""
        self.cfg = cfg
        self._keep = []
        L = cfg.layers
        self.cross = all(n in layer_weights[0] for n in CROSS_TENSORS)
        arrays = {}
        for name in list(LAYER_TENSORS) + (list(CROSS_TENSORS) if self.cross else []):
            arr = (P * L)()
            for l in range(L):
                a = np.ascontiguousarray(layer_weights[l][name])
                self._keep.append(a)
                arr[l] = a.ctypes.data
            arrays[name] = arr
        self._keep += [arrays]
        g = [np.ascontiguousarray(x) for x in (final_norm, embedding, w_head, s_head)]
        self._keep += g
        cross = [_c.cast(arrays[n], _c.POINTER(P)) if self.cross else None for n in CROSS_TENSORS]
        self.s = _Decoder(cfg.layers, cfg.dim, cfg.heads, cfg.head_dim, cfg.ffn, cfg.vocab, cfg.rope_theta, 1e-6,
                          *[_c.cast(arrays[n], _c.POINTER(P)) for n in LAYER_TENSORS],
                          *[x.ctypes.data for x in g], *cross)
        self.capacity = capacity
        self.cos, self.sin = rope_tables(cfg.rope_theta, cfg.head_dim, capacity)

    def cross_memory(self, memory):
        """memory fp32 [frames][dim] -> int8 K/V [layers][frames][width] + scales."""
        c = self.cfg
        memory = f32(memory)
        frames, W = memory.shape[0], c.heads * c.head_dim
        out = {"k": np.zeros((c.layers, frames, W), np.int8), "v": np.zeros((c.layers, frames, W), np.int8),
               "ks": np.zeros((c.layers, frames, c.heads), np.float32),
               "vs": np.zeros((c.layers, frames, c.heads), np.float32)}
        for l in range(c.layers):
            st = lib().ndo_cross_memory(_c.byref(self.s), l, ptr(memory), frames, ptr(out["k"][l]),
                                        ptr(out["v"][l]), ptr(out["ks"][l]), ptr(out["vs"][l]))
            if st != 0:
                raise MemoryError("oracle scratch allocation failed")
        return out

    def new_kv(self):
        c = self.cfg
        W = c.heads * c.head_dim
        return {"k": np.zeros((c.layers, self.capacity, W), np.int8),
                "v": np.zeros((c.layers, self.capacity, W), np.int8),
                "ks": np.zeros((c.layers, self.capacity, c.heads), np.float32),
                "vs": np.zeros((c.layers, self.capacity, c.heads), np.float32)}

    def row(self, token, pos, kv, memory=None):
        logits = np.empty(self.cfg.vocab, np.float32)
        if memory is None:
            st = lib().ndo_decoder_row(_c.byref(self.s), token, pos, self.capacity, ptr(kv["k"]), ptr(kv["v"]),
                                       ptr(kv["ks"]), ptr(kv["vs"]), ptr(self.cos), ptr(self.sin), ptr(logits))
        else:
            frames = memory["k"].shape[1]
            st = lib().ndo_decoder_row_cross(_c.byref(self.s), token, pos, self.capacity, ptr(kv["k"]),
                                             ptr(kv["v"]), ptr(kv["ks"]), ptr(kv["vs"]), ptr(self.cos),
                                             ptr(self.sin), frames, ptr(memory["k"]), ptr(memory["v"]),
                                             ptr(memory["ks"]), ptr(memory["vs"]), ptr(logits))
        if st != 0:
            raise MemoryError("oracle scratch allocation failed")
        return logits


def beam_search(dec, memory, prompt, width, max_steps, eos, length_penalty=1.0, mask_special_023=True):
    """Whistle.BeamSearch (src/Needle/Whistle.Decode.cs:224-350) on the oracle
    decoder: per step every live beam's logits give its top-`width`
    (TopKLogSoftmax, ids 0/2/3 masked), candidates = beam score + log-prob
    (fp32), sorted by score (descending; equal scores keep (beam, rank)
    order), EOS candidates join `finished`, at most `width` others stay live;
    stop when nothing is kept, or when `width` have finished and the best
    normalised finished score (score / (len+1)^penalty) is at least the best
    normalised live one; winner = best finished, else best live
    (score / len^penalty).  Returns (tokens, normalised score)."""
    c = dec.cfg

    def normalized(score, length):
        if length_penalty == 0:
            return np.float32(score)
        return np.float32(score) / np.float32(np.power(np.float32(length), np.float32(length_penalty)))

    kv = dec.new_kv()
    logits = None
    for pos, tok in enumerate(prompt):
        logits = dec.row(int(tok), pos, kv, memory)
    live = [(kv, len(prompt), logits)]
    live_tokens = [[]]
    live_scores = [np.float32(0.0)]
    finished = []
    for _ in range(max_steps):
        cands = []
        for i, (_, _, lg) in enumerate(live):
            idx, lp, _ = topk_logsoftmax(lg, width, mask_special_023=mask_special_023, want_probs=False)
            for k in range(width):
                cands.append((np.float32(live_scores[i] + lp[k]), i, int(idx[k]), len(cands)))
        cands.sort(key=lambda t: (-t[0], t[3]))
        kept = []
        for sc, parent, tok, _ in cands:
            if tok == eos:
                finished.append((sc, list(live_tokens[parent])))
            else:
                kept.append((sc, parent, tok))
            if len(kept) >= width:
                break
        if not kept:
            break
        if len(finished) >= width:
            best_f = max(normalized(s, len(t) + 1) for s, t in finished)
            best_l = max(normalized(s, len(live_tokens[p]) + 1) for s, p, _ in kept)
            if best_f >= best_l:
                break
        new_live, new_tokens, new_scores = [], [], []
        for sc, parent, tok in kept:
            pkv, ppos, _ = live[parent]
            ckv = {k: v.copy() for k, v in pkv.items()}
            lg = dec.row(tok, ppos, ckv, memory)
            new_live.append((ckv, ppos + 1, lg))
            new_tokens.append(live_tokens[parent] + [tok])
            new_scores.append(sc)
        live, live_tokens, live_scores = new_live, new_tokens, new_scores
    best, best_score = None, -np.inf
    for sc, toks in finished:
        v = normalized(sc, len(toks) + 1)
        if v > best_score:
            best, best_score = toks, v
    if best is not None:
        return best, float(best_score)
    for sc, toks in zip(live_scores, live_tokens):
        v = normalized(sc, len(toks))
        if v > best_score:
            best, best_score = toks, v
    return (best or []), float(best_score)


# ---------------------------------------------------------------- AVX2 --
# The CPU baseline (oracle/avx2_decoder.c): the reference's AVX2 kernels'
# algorithms on all host cores, equal to the scalar restatement bit for bit.

def host_threads():
    """Threads for the CPU baseline: NEEDLE_THREADS when set (the reference's
    thread-count variable), else every host core."""
    return int(os.environ.get("NEEDLE_THREADS", "0")) or os.cpu_count() or 1


def matmul_i8g32_avx2(q, sa, w, sw, threads=None):
    q = np.ascontiguousarray(q, np.int8)
    sa = f32(sa)
    w = np.ascontiguousarray(w, np.int8)
    sw = np.ascontiguousarray(sw, np.uint16)
    m, k = q.shape
    n = w.shape[0]
    y = np.empty((m, n), np.float32)
    lib().ndb_matmul_i8g32(ptr(w), ptr(sw), n, k, ptr(q), ptr(sa), m, ptr(y), n, threads or host_threads())
    return y


class AVX2Linear:
    """A prepared int8 linear for repeated timing."""

    def __init__(self, w, sw):
        self.w = np.ascontiguousarray(w, np.int8)
        self.sw = np.ascontiguousarray(sw, np.uint16)
        self.n, self.k = self.w.shape
        self.h = lib().ndb_linear_create(ptr(self.w), ptr(self.sw), self.n, self.k)
        if not self.h:
            raise MemoryError("AVX2 linear allocation failed")

    def run(self, q, sa, y, threads=None):
        lib().ndb_linear_run(self.h, ptr(q), ptr(sa), q.shape[0], ptr(y), y.shape[1], threads or host_threads())

    def close(self):
        if self.h:
            lib().ndb_linear_destroy(self.h)
            self.h = None


class AVX2Decoder:
    """The decoder's batched decode step on the CPU with AVX2 and all host
    cores (ndb_decode_step), over the tensors of an oracle Decoder."""

    def __init__(self, dec):
        self.dec = dec
        self.h = lib().ndb_model_create(_c.byref(dec.s))
        if not self.h:
            raise MemoryError("AVX2 model allocation failed")

    def step(self, tokens, positions, kvs, threads=None):
        """tokens/positions [rows]; kvs: one new_kv() dict per row.  Writes
        each row's K/V at its position and returns logits [rows][vocab]."""
        rows = len(tokens)
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(positions, np.int32)
        arrs = {key: (P * rows)(*[kv[key].ctypes.data for kv in kvs]) for key in ("k", "v", "ks", "vs")}
        logits = np.empty((rows, self.dec.cfg.vocab), np.float32)
        st = lib().ndb_decode_step(self.h, rows, ptr(t), ptr(p), self.dec.capacity, arrs["k"], arrs["v"],
                                   arrs["ks"], arrs["vs"], ptr(self.dec.cos), ptr(self.dec.sin), ptr(logits),
                                   threads or host_threads())
        if st != 0:
            raise MemoryError("AVX2 step scratch allocation failed")
        return logits

    def close(self):
        if self.h:
            lib().ndb_model_destroy(self.h)
            self.h = None


# ------------------------------------------------------------ synthetic --
# The benchmark configs' inputs built on the host by the oracle's own copy of
# the generator (no CUDA library involved): the synthetic decoder's tensors
# and the prefix K/V of its sessions.  Stream ids under the model seed:
# embedding 1, final norm 2, layer l field f at 100 + 16*l + f (w_qkv, s_qkv,
# w_o, s_o, w_gu, s_gu, w_d, s_d, attn_norm, ffn_norm); weights U{-127..127},
# scales fp16 U(0.001, 0.02), norms 1 + 0.1*normal, the embedding fp16
# 0.02*normal, the head int8 quantized from the embedding per (row, 32-group).

def synth_normal(seed, stream, count, scale=1.0, first=0):
    out = np.empty(count, np.float32)
    lib().ndo_synth_normal(seed, stream, first, count, scale, ptr(out))
    return out


def synth_normal_f16(seed, stream, count, scale=1.0, first=0):
    """fp16 bits (IEEE round to nearest even) of normal * scale."""
    return synth_normal(seed, stream, count, scale, first).astype(np.float16).view(np.uint16)


def synth_uniform_f16(seed, stream, count, lo, hi, first=0):
    out = np.empty(count, np.float32)
    lib().ndo_synth_uniform(seed, stream, first, count, lo, hi, ptr(out))
    return out.astype(np.float16).view(np.uint16)


def synth_int8(seed, stream, count, first=0):
    out = np.empty(count, np.int8)
    lib().ndo_synth_int8(seed, stream, first, count, ptr(out))
    return out


class DecoderConfig:
    """The synthetic decoder's shape (defaults: the 12-layer decoder of
    configs 2, 3 and 5)."""

    def __init__(self, layers=12, dim=512, heads=8, head_dim=64, ffn=2048, vocab=8192, rope_theta=10000.0, seed=1):
        self.layers, self.dim, self.heads, self.head_dim = layers, dim, heads, head_dim
        self.ffn, self.vocab, self.rope_theta, self.seed, self.cross = ffn, vocab, rope_theta, seed, 0


_FIELDS = ["w_qkv", "s_qkv", "w_o", "s_o", "w_gu", "s_gu", "w_d", "s_d", "attn_norm", "ffn_norm"]


def synthetic_decoder(cfg, capacity):
    """An oracle Decoder over the synthetic decoder's tensors."""
    seed, d, F, V = cfg.seed, cfg.dim, cfg.ffn, cfg.vocab
    G, GF = d // 32, F // 32
    shapes = {"w_qkv": (3 * d * d, "i8"), "s_qkv": (3 * d * G, "s"), "w_o": (d * d, "i8"), "s_o": (d * G, "s"),
              "w_gu": (2 * F * d, "i8"), "s_gu": (2 * F * G, "s"), "w_d": (d * F, "i8"), "s_d": (d * GF, "s"),
              "attn_norm": (d, "n"), "ffn_norm": (d, "n")}

    def gen(name, stream):
        count, kind = shapes[name]
        if kind == "i8":
            return synth_int8(seed, stream, count)
        if kind == "s":
            return synth_uniform_f16(seed, stream, count, 0.001, 0.02)
        return (np.float32(1.0) + np.float32(0.1) * synth_normal(seed, stream, count)).astype(np.float32)

    layers = [{name: gen(name, 100 + 16 * l + f) for f, name in enumerate(_FIELDS)} for l in range(cfg.layers)]
    final_norm = (np.float32(1.0) + np.float32(0.1) * synth_normal(seed, 2, d)).astype(np.float32)
    emb = synth_normal_f16(seed, 1, V * d, scale=0.02)
    e = emb.view(np.float16).astype(np.float32).reshape(V, d // 32, 32)
    peak = np.abs(e).max(axis=2)
    s16 = np.where(peak > 0, peak / np.float32(127.0), np.float32(1.0)).astype(np.float32).astype(np.float16)
    inv = (np.float32(1.0) / s16.astype(np.float32)).astype(np.float32)
    w_head = np.clip(np.rint(e * inv[:, :, None]), -127, 127).astype(np.int8).reshape(-1)
    s_head = s16.view(np.uint16).reshape(-1)
    return Decoder(cfg, layers, final_norm, emb, w_head, s_head, capacity)


def synthetic_prefix_kv(dec, kv, count, seed, session):
    """Positions [0, count) of a session's cache: fp16 N(0,1) K and V from
    (seed, session) at index ((((layer*2 + kind) << 20) + pos) * heads +
    head) * 64 + d, quantized per (position, head) (QuantizeInt8)."""
    H = dec.cfg.heads
    for layer in range(dec.cfg.layers):
        for kind, (vals, scales) in enumerate((("k", "ks"), ("v", "vs"))):
            first = ((layer * 2 + kind) << 20) * H * 64
            raw = synth_normal_f16(seed, session, count * H * 64, first=first)
            q, sc = quantize_rows(raw.view(np.float16).astype(np.float32).reshape(count * H, 64))
            kv[vals][layer, :count] = q.reshape(count, H * 64)
            kv[scales][layer, :count] = sc.reshape(count, H)
