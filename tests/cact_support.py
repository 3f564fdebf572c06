"""Writes small synthetic Needle-3 archives (.cact) for the loader tests.

The layout is the reference's (src/Needle/Model.cs:191-198, 307-361):
 * a 196-byte header of uint32 words (magic, record count, codebook entries,
   then the Geometry words 3..48, word 48 the fp32 RoPE theta);
 * the codebook levels (fp32);
 * the record table (44-byte records: dtype, ndim, pad, 4 shape words,
   offset, bytes, group, bits);
 * the tensor bytes, with the tokenizer blob as the last record.
Tensors follow the Reader's order: embedding, each layer (LayerWeights + MlpWeights),
the hyper-connections, the Engram sites, the final norm, then either probe
heads (manifest + ProbeHead) or an audio section.  Shapes are small and
only as constrained as the loader checks them.
"""
import struct

import numpy as np

MAGIC = 0x05E12A84
HEADER_BYTES = 196
FP16, FP32, CQ, RAW = 1, 2, 3, 4

GEOMETRY = dict(kv_window=64, vocab=256, dim=128, heads=2, kv_heads=1, layers=2, qk_dim=48, v_dim=64, max_seq=512,
                hada_n=128, lanes=4, sliding_window=64, global_mask=0b10, conv_taps=3, engram_slots=97,
                engram_sub=1, engram_tables=4, engram_conv_taps=4, engram_dilation=2, engram_seed_heads=2,
                orders=[2, 3], sites=[1], rope_theta=10000.0)
WORDS = dict(kv_window=3, vocab=5, dim=7, heads=8, kv_heads=9, layers=10, qk_dim=11, v_dim=12, max_seq=13, hada_n=14,
             lanes=15, sliding_window=16, conv_taps=19, engram_slots=20, engram_sub=21, engram_tables=22,
             engram_conv_taps=23, engram_dilation=24, engram_seed_heads=25)

LAYER = ["layer.norm_in", ("layer.q", 96), ("layer.k", 48), ("layer.v", 64), "layer.q_taps", "layer.k_taps",
         "layer.v_taps", "layer.q_norm", "layer.k_norm", ("layer.gate", 128), ("layer.out", 128), "layer.post_norm",
         "layer.attn_gate", "layer.pre_hada"] + ["layer.mlp." + n for n in (
             "d1", "d2", "b2", "d3", "d4", "w1a", "w1b", "w2a", "w2b", "w3a", "w3b", "cond_v", "cond_u")]


def half_to_single(halves, exact=True):
    """Scalar.HalfToSingle / HalfToSingleUpstream (src/Needle/Scalar.cs:113-128) on uint16 words."""
    h = np.asarray(halves, np.uint16).astype(np.uint32)
    mag = h & 0x7FFF
    bits = ((mag << 13) + 0x38000000) | ((h & 0x8000) << 16)
    out = bits.astype(np.uint32).view(np.float32).copy()
    if exact:
        sub = (mag > 0) & (mag < 0x400)
        v = mag[sub].astype(np.float32) * np.float32(5.9604645e-8)
        out[sub] = np.where(h[sub] & 0x8000, -v, v)
    out[mag == 0] = 0.0
    return out


class Archive:
    """Collects records in order; ``build()`` returns the archive bytes."""

    def __init__(self, seed=0, geometry=None):
        self.rng = np.random.default_rng(seed)
        self.g = dict(GEOMETRY, **(geometry or {}))
        self.records = []  # (role, index, dtype, shape, payload bytes, bits, expected)
        levels = np.zeros(28, np.float32)
        levels[0:4] = [-1.5, -0.5, 0.5, 1.5]
        levels[12:28] = np.linspace(-2.0, 2.0, 16).astype(np.float32) * 0.75
        self.levels = levels

    def dense(self, role, index, n, fp16=True, values=None):
        if fp16:
            raw = (np.asarray(values, np.uint16) if values is not None
                   else self.rng.normal(0, 1, n).astype(np.float16).view(np.uint16))
            self.records.append((role, index, FP16, [raw.size], raw.tobytes(), 0, ("dense16", raw)))
        else:
            v = np.asarray(values, np.float32) if values is not None else self.rng.normal(0, 1, n).astype(np.float32)
            self.records.append((role, index, FP32, [v.size], v.tobytes(), 0, ("dense32", v)))

    def cq(self, role, index, rows, cols, bits):
        codes = self.rng.integers(0, 256, rows * cols * bits // 8, dtype=np.uint8)
        norms = self.rng.uniform(0.01, 0.2, rows * (cols // 128)).astype(np.float16).view(np.uint16)
        self.records.append((role, index, CQ, [rows, cols], codes.tobytes() + norms.tobytes(), bits,
                             ("cq", codes, norms, rows, cols, bits)))

    def perm(self, role, n, values=None):
        p = np.asarray(values if values is not None else self.rng.permutation(n), np.float32)
        self.records.append((role, 0, FP32, [p.size], p.tobytes(), 0, ("perm", p.astype(np.int32))))

    def raw(self, payload):
        self.records.append(("tokenizer", 0, RAW, [len(payload)], payload, 0, ("raw", payload)))

    def standard(self, probe_codes=(2,), audio=False, final_norm=None):
        """A full archive in the Reader's order."""
        g = self.g
        d = g["dim"]
        self.cq("embedding", 0, g["vocab"], d, 4)
        for layer in range(g["layers"]):
            for item in LAYER:
                if isinstance(item, tuple):
                    self.cq(item[0], layer, item[1], d, 2)
                elif item == "layer.attn_gate":
                    self.dense(item, layer, 1, fp16=False)
                else:
                    self.dense(item, layer, self._layer_size(item), fp16=layer % 2 == 0)
        for n in ("a_pre", "a_post", "a_res", "b_pre", "b_post", "b_res"):
            self.dense("hyper." + n, 0, 16)
        for n in ("phi_pre", "phi_post", "phi_res"):
            self.cq("hyper." + n, 0, 24, 4 * d, 2)
        if g["hada_n"] > 0:
            self.perm("hyper.perm_a", g["hada_n"])
            self.perm("hyper.perm_b", g["hada_n"])
        for s in range(len(g["sites"])):
            sub = g["engram_sub"] if g["engram_sub"] % 128 == 0 else d  # tables tile the input when sub allows
            self.cq("site.tables", s, g["engram_tables"] * g["engram_slots"], sub, 4)
            self.cq("site.key", s, d, d, 2)
            self.cq("site.value", s, d, d, 2)
            self.dense("site.taps", s, 4 * d)
        if final_norm is not None:
            self.dense("final_norm", 0, None, values=final_norm)
        else:
            self.dense("final_norm", 0, d)
        if audio:
            self.dense("audio", 0, 13, fp16=False)
            self.cq("audio", 1, 8, d, 4)
            self.dense("audio", 2, 40)
        elif probe_codes:
            self.dense("manifest", 0, None, fp16=False, values=np.array(probe_codes, np.float32))
            for h, code in enumerate(probe_codes):
                rows = g["layers"] + 1
                self.cq("probe.probe_vectors", h, rows * 2, d, 4)
                self.dense("probe.gain", h, rows * 2)
                self.cq("probe.query_vectors", h, 2, d, 4)
                self.dense("probe.row_bias", h, 2 * rows * 2)
                self.cq("probe.projection", h, 1, 2 * d, 4)
                self.dense("probe.bias", h, 1)
                if code == 3:
                    self.dense("probe.router", h, 5)
        self.raw(b"needle tokenizer blob \x00\x01\x02")
        return self

    def _layer_size(self, role):
        """Sizes of the MLP factors for the HadaRows x HadaCols split (HadamardMlp.Apply), else 24."""
        g = self.g
        d, width = g["dim"], g["hada_n"]
        rows = 1 << ((width - 1).bit_length() // 2) if width > 0 else 1
        cols = width // rows if width > 0 else 1
        in_rows = (d + cols - 1) // cols
        sizes = {"d1": d, "d2": width, "b2": width, "d3": width, "d4": d, "w1a": in_rows * rows, "w1b": cols * cols,
                 "w2a": rows * rows, "w2b": cols * cols, "w3a": rows * rows, "w3b": cols * cols, "cond_v": d * 8,
                 "cond_u": 8 * width}
        if role == "layer.pre_hada":
            return d
        return sizes.get(role.rsplit(".", 1)[1], 24) if role.startswith("layer.mlp.") else 24

    def header_words(self):
        g = self.g
        h = np.zeros(HEADER_BYTES // 4, np.uint32)
        h[0], h[1], h[2] = MAGIC, len(self.records), self.levels.size
        for k, w in WORDS.items():
            h[w] = g[k]
        h[17], h[18] = g["global_mask"] & 0xFFFFFFFF, g["global_mask"] >> 32
        h[26] = len(g["orders"])
        h[27:27 + len(g["orders"])] = g["orders"]
        h[31] = len(g["sites"])
        h[32:32 + len(g["sites"])] = g["sites"]
        h[48] = np.array([g["rope_theta"]], np.float32).view(np.uint32)[0]
        return h

    def build(self, header=None):
        h = self.header_words() if header is None else header
        table_at = HEADER_BYTES + self.levels.size * 4
        at = table_at + 44 * len(self.records)
        table, blobs = b"", b""
        for _, _, dtype, shape, payload, bits, _ in self.records:
            at = (at + 15) // 16 * 16
            pad = at - (table_at + 44 * len(self.records) + len(blobs))
            blobs += b"\x00" * pad
            shape4 = list(shape) + [0] * (4 - len(shape))
            table += struct.pack("<BBH4IQQII", dtype, len(shape), 0, *shape4, at, len(payload),
                                 128 if dtype == CQ else 0, bits)
            blobs += payload
            at += len(payload)
        return h.tobytes() + self.levels.tobytes() + table + blobs


def needle3_decoder_archive(seed=0, **geometry):
    """A complete Needle-3 archive whose shapes drive a whole decode step
    (the phi matrices cover every layer, the projections have their head
    shapes) with tame values: unit-scale norms near zero, small conv taps
    and MLP factors, so activations stay finite through the layers."""
    g = dict(GEOMETRY, dim=512, heads=2, kv_heads=1, qk_dim=48, v_dim=64, layers=2, vocab=384, hada_n=512,
             engram_sub=128, engram_tables=4, engram_slots=97, orders=[2, 3], sites=[1], sliding_window=8,
             global_mask=0b10, max_seq=512)
    g.update(geometry)
    a = Archive(seed=seed, geometry=g)
    rng = a.rng
    d, L = g["dim"], g["layers"]
    qw, kw, vw, ow = g["heads"] * g["qk_dim"], g["kv_heads"] * g["qk_dim"], g["kv_heads"] * g["v_dim"], \
        g["heads"] * g["v_dim"]

    def small(n, sd):
        return rng.normal(0, sd, n).astype(np.float16).view(np.uint16)

    a.cq("embedding", 0, g["vocab"], d, 4)
    sizes = {"layer.norm_in": d, "layer.q_taps": 3 * qw, "layer.k_taps": 3 * kw, "layer.v_taps": 3 * vw,
             "layer.q_norm": g["qk_dim"], "layer.k_norm": g["qk_dim"], "layer.post_norm": d, "layer.pre_hada": d}
    shapes = {"layer.q": (qw, d), "layer.k": (kw, d), "layer.v": (vw, d), "layer.gate": (ow, d), "layer.out": (d, ow)}
    for layer in range(L):
        for item in LAYER:
            role = item[0] if isinstance(item, tuple) else item
            if role in shapes:
                a.cq(role, layer, shapes[role][0], shapes[role][1], 2)
            elif role == "layer.attn_gate":
                a.dense(role, layer, 1, fp16=False, values=rng.normal(0, 1, 1).astype(np.float32))
            elif role.startswith("layer.mlp."):
                n = a._layer_size(role)
                sd = 0.1 if role.rsplit(".", 1)[1].startswith(("w", "cond")) else 0.3
                a.dense(role, layer, n, values=small(n, sd))
            else:
                sd = 0.5 if role.endswith("taps") else 0.1
                a.dense(role, layer, sizes[role], values=small(sizes[role], sd))
    for n, count in (("a_pre", L), ("a_post", L), ("a_res", L), ("b_pre", 4 * L), ("b_post", 4 * L),
                     ("b_res", 16 * L)):
        a.dense("hyper." + n, 0, count, values=small(count, 0.5))
    for n, rows in (("phi_pre", 4 * L), ("phi_post", 4 * L), ("phi_res", 16 * L)):
        a.cq("hyper." + n, 0, rows, 4 * d, 4)
    a.perm("hyper.perm_a", g["hada_n"])
    a.perm("hyper.perm_b", g["hada_n"])
    for s in range(len(g["sites"])):
        a.cq("site.tables", s, g["engram_tables"] * g["engram_slots"], g["engram_sub"], 4)
        a.cq("site.key", s, d, d, 2)
        a.cq("site.value", s, d, d, 2)
        a.dense("site.taps", s, 4 * d, values=small(4 * d, 0.3))
    a.dense("final_norm", 0, d, values=small(d, 0.1))
    a.raw(b"needle tokenizer blob \x00\x01\x02")
    return a


MLP_NAMES = ("d1", "d2", "b2", "d3", "d4", "w1a", "w1b", "w2a", "w2b", "w3a", "w3b", "cond_v", "cond_u")


def mel_bank(fft, mels, rate):
    """A triangular mel filterbank [fft/2 + 1][mels] (nonnegative, each bin
    in at most two adjacent filters), fp32."""
    def hz_to_mel(f):
        return 2595.0 * np.log10(1.0 + f / 700.0)

    bins = fft // 2 + 1
    edges = 700.0 * (10 ** (np.linspace(hz_to_mel(0.0), hz_to_mel(rate / 2), mels + 2) / 2595.0) - 1.0)
    freqs = np.linspace(0, rate / 2, bins)
    bank = np.zeros((bins, mels), np.float32)
    for m in range(mels):
        lo, mid, hi = edges[m], edges[m + 1], edges[m + 2]
        up = (freqs - lo) / (mid - lo)
        down = (hi - freqs) / (hi - mid)
        bank[:, m] = np.maximum(0.0, np.minimum(up, down)).astype(np.float32)
    return bank


def whistle_archive(seed=0, encoder_layers=2, conv_kernel=7, stem_width=128, mels=80, fft=512, window=400, hop=160,
                    sample_rate=16000, **geometry):
    """A Needle-3 archive with a Whistle audio section in AudioWeights' order
    (src/Needle/Audio.cs:117-149): the 13-entry manifest; per decoder layer
    the CrossWeights (norm, Q, K, V, gate, out, q/k norms, post norm, mix
    logit); the position-mix logit; per encoder layer the EncoderLayer (six
    norms, Q/K/V/gate/out, q/k norms, attention gate logit, the two pointwise
    convs, the depthwise taps, two MlpWeights); the encoder's
    HyperConnections (no permutations); the final norm; the three-stage stem
    (first 3x3 conv, depthwise + pointwise twice, the output projection);
    the mel filterbank.  Values are tame (norm scales near zero, small conv
    taps and MLP factors) so activations stay finite through the encoder."""
    a = needle3_decoder_archive(seed=seed, **geometry)
    a.records.pop()  # the tokenizer goes last again below
    g, rng = a.g, a.rng
    d, L, E, s = g["dim"], g["layers"], encoder_layers, stem_width
    H, KV, QK, VD = g["heads"], g["kv_heads"], g["qk_dim"], g["v_dim"]
    qw, kw, vw, ow = H * QK, KV * QK, KV * VD, H * VD
    g.update(encoder_layers=E, conv_kernel=conv_kernel, stem_width=s, mels=mels, fft=fft, window=window, hop=hop,
             sample_rate=sample_rate)
    k = [0]

    def small(n, sd):
        return rng.normal(0, sd, n).astype(np.float16).view(np.uint16)

    def dense(n, sd=None, values=None, fp16=True):
        if values is None:
            values = small(n, sd) if fp16 else rng.normal(0, sd, n).astype(np.float32)
        a.dense("audio", k[0], n, fp16=fp16, values=values)
        k[0] += 1

    def cq(rows, cols, bits=2):
        a.cq("audio", k[0], rows, cols, bits)
        k[0] += 1

    manifest = np.zeros(13, np.float32)
    manifest[3:13] = [E, 4, conv_kernel, s, 3, mels, sample_rate, fft, window, hop]
    dense(13, values=manifest, fp16=False)
    for _ in range(L):  # CrossWeights
        dense(d, 0.1)
        cq(H * QK, d)
        cq(H * QK, d)
        cq(H * VD, d)
        cq(H * VD, d)
        cq(d, H * VD)
        dense(QK, 0.1)
        dense(QK, 0.1)
        dense(d, 0.1)
        dense(1, 1.0, fp16=False)
    dense(1, 1.0, fp16=False)  # position mix logit
    for _ in range(E):  # EncoderLayer
        for _ in range(6):
            dense(d, 0.1)
        cq(qw, d)
        cq(kw, d)
        cq(vw, d)
        cq(ow, d)
        cq(d, ow)
        dense(QK, 0.1)
        dense(QK, 0.1)
        dense(1, 1.0, fp16=False)  # attention gate logit
        cq(2 * d, d)
        cq(d, d)
        dense(conv_kernel * d, 0.3)
        for _ in range(2):  # MlpWeights
            for n in MLP_NAMES:
                size = a._layer_size("layer.mlp." + n)
                dense(size, 0.1 if n.startswith(("w", "cond")) else 0.3)
    for n, count in (("a_pre", E), ("a_post", E), ("a_res", E), ("b_pre", 4 * E), ("b_post", 4 * E),
                     ("b_res", 16 * E)):
        dense(count, 0.5)
    cq(4 * E, 4 * d, 4)
    cq(4 * E, 4 * d, 4)
    cq(16 * E, 4 * d, 4)
    dense(d, 0.1)  # final norm
    dense(9 * s, 0.3)  # stem first
    dense(9 * s, 0.3)  # stem depthwise 1
    cq(s, s)
    dense(9 * s, 0.3)  # stem depthwise 2
    cq(s, s)
    cq(d, 10 * s)  # stem out
    dense(None, values=mel_bank(fft, mels, sample_rate).reshape(-1), fp16=False)
    a.raw(b"needle tokenizer blob \x00\x01\x02")
    return a
