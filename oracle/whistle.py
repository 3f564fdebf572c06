"""CPU restatement of the Whistle encoder: Whistle.Encode and BuildCrossMemory
(src/Needle/Whistle.cs:179-200, 886-914), the reference's scalar tier
throughout (Simd.Enabled false: MathF.Exp and MathF.Log correctly rounded,
no fused multiply-adds, the plain radix-2 FFT).

TEST INFRASTRUCTURE ONLY.  The checker for the device encoder in the
library; never imported by the library.  The front end is whistle_oracle.c;
every other operation is a call of needle_oracle.c's restatement of the
reference routine or a numpy float32 elementwise step (one IEEE rounding per
operation, as the scalar C# loops):

  Encode (:179-200)
    FeatureJob (Frontend.cs:82-130): per frame of `hop` samples the Hann-
    windowed FFT power spectrum, mel sums, the peak; log(x + floor) with
    floor = max(peak * 1e-8, 1e-30); Normalize per mel column in double
    Stem (:282-299, 346-470): three stages at strides 2 in time and
    frequency; stage 1 a 3x3 conv from the mel plane to StemWidth channels
    (AddScaled) and SiLU; stages 2 and 3 a depthwise 3x3 conv
    (MultiplyAccumulate), a 2-bit CQ pointwise matmul per (row, frequency)
    and SiLU; the 10 x StemWidth plane transposed to channel-major and the
    StemOut CQ matmul to Dim
    RunEncoder (:794-828), per layer: RmsUnit of the 4-lane stream and a
    4-bit Prepare; the layer's phi slices; gates, Mix4 and Sinkhorn4x4
    (ExecutePreHyper); MLP0 (scale 0.5); self-attention over all frames
    (ZeroCenteredRms, the Q/K/V/gate matmuls, per-head norms, RoPE at the
    frame index, int8 quantization, AttentionHead over [0, frames),
    MultiplyBySigmoid by the gate, the out matmul, PostNormAdd); the
    convolution module (ZeroCenteredRms, Pw1, Glu, the depthwise conv over
    time with ConvKernel taps, ZeroCenteredRms, SiLU, Pw2, residual add);
    MLP (scale 0.5); CombineDiff4x4.  Then Mix4 by 1/4 and ZeroCenteredRms
    with the final norm.
  BuildCrossMemory (:886-914): the encoder rows plus PositionMix times the
  sin / cos position tables, FakeA8, a 2-bit Prepare; per decoder layer the
  cross K and V matmuls, ZeroCenteredRms of each head's key, int8
  quantization per (frame, head).
"""
import ctypes

import numpy as np

from . import oracle as O

MLP = ("d1", "d2", "b2", "d3", "d4", "w1a", "w1b", "w2a", "w2b", "w3a", "w3b", "cond_v", "cond_u")
CROSS = ("norm", "q", "k", "v", "gate", "out", "q_norm", "k_norm", "post_norm", "mix")
ENCODER = ("pre_mlp_norm0", "attn_norm", "post_attn_norm", "conv_norm", "conv_out_norm", "pre_mlp_norm", "q", "k",
           "v", "gate", "out", "q_norm", "k_norm", "attn_gate", "pw1", "pw2", "depthwise") + \
    tuple("mlp0." + n for n in MLP) + tuple("mlp." + n for n in MLP)
HYPER = ("a_pre", "a_post", "a_res", "b_pre", "b_post", "b_res", "phi_pre", "phi_post", "phi_res")
TAIL = ("final_norm", "stem_first", "stem_depthwise1", "stem_pointwise1", "stem_depthwise2", "stem_pointwise2",
        "stem_out", "mel")
LANES = 4


def audio_layout(decoder_layers, encoder_layers):
    """Index of each audio record in AudioWeights' reading order
    (src/Needle/Audio.cs:117-149); the manifest is record 0."""
    names = ["manifest"]
    for l in range(decoder_layers):
        names += [f"cross{l}.{n}" for n in CROSS]
    names.append("position_mix")
    for l in range(encoder_layers):
        names += [f"enc{l}.{n}" for n in ENCODER]
    names += ["hyper." + n for n in HYPER]
    names += list(TAIL)
    return {n: k for k, n in enumerate(names)}


def _f(a):
    return np.ascontiguousarray(a, np.float32)


def _p(a):
    return a.ctypes.data


class WhistleOracle:
    """`dense(role, i)` -> float32 array, `cq(role, i)` -> (codes [rows][cols*bits/8]
    uint8, norms [rows][cols/128] uint16, rows, cols, bits), `perm(role)` ->
    int32 array, `info` the geometry dict of ndl_model_get_info, `levels` the
    codebook's 28 levels; the audio tensors are role "audio"."""

    def __init__(self, info, levels, dense, cq, perm):
        self.g = info
        self.dense, self.cq, self.perm = dense, cq, perm
        self.book2 = O.codebook(np.asarray(levels[0:4], np.float32), 4)
        self.book4 = O.codebook(np.asarray(levels[12:28], np.float32), 16)
        manifest = _f(dense("audio", 0))
        (self.encoder_layers, self.lanes, self.conv_kernel, self.stem_width, stages, self.mels, self.rate, self.fft,
         self.window, self.hop) = [int(round(float(v))) for v in manifest[3:13]]
        assert stages == 3, "three-stage stem expected"
        self.at = audio_layout(info["layers"], self.encoder_layers)
        self.dim = info["dim"]

    def A(self, name):
        return _f(self.dense("audio", self.at[name]))

    def _mm(self, name, act, rows=None):
        codes, norms, nrows, cols, bits = self.cq("audio", self.at[name])
        vals, sc, off, _ = act
        book = self.book2 if bits == 2 else self.book4
        r0, r1 = (0, nrows) if rows is None else rows
        y = np.zeros((vals.shape[0], nrows), np.float32)
        O.matmul_rows_cq(codes, norms, book, bits, vals, sc, off, r0, r1, y)
        return y[:, r0:r1].copy()

    # -- front end --
    def features(self, pcm):
        """(frames l0, normalized log-mel features [l0][mels])."""
        lib = O.lib()
        pcm = _f(pcm)
        samples = min(pcm.size, 30 * self.rate)
        l0 = samples // self.hop
        if l0 < 1:
            return 0, np.zeros((0, self.mels), np.float32)
        fft, window, mels, half = self.fft, self.window, self.mels, self.window // 2
        padded = np.zeros(half + samples + half + self.hop + fft, np.float32)
        padded[half:half + samples] = pcm[:samples]
        bank = self.A("mel")
        hann, cosines, sines = (np.zeros(window, np.float32), np.zeros(fft // 2, np.float32),
                                np.zeros(fft // 2, np.float32))
        bitrev, first, count = (np.zeros(fft, np.int32), np.zeros(fft // 2 + 1, np.int32),
                                np.zeros(fft // 2 + 1, np.int32))
        lib.ndo_frontend_tables(fft, window, _p(bank), mels, _p(hann), _p(cosines), _p(sines), _p(bitrev), _p(first),
                                _p(count))
        out = np.zeros((l0, mels), np.float32)
        peak = np.float32(0.0)
        for frame in range(l0):
            seg = ctypes.c_void_p(padded.ctypes.data + frame * self.hop * 4)
            p = lib.ndo_mel_frame(seg, fft, window, _p(hann), _p(cosines), _p(sines), _p(bitrev), _p(bank), mels,
                                  _p(first), _p(count), _p(out[frame]))
            peak = max(peak, np.float32(p))
        floor = max(np.float32(peak * np.float32(1e-8)), np.float32(1e-30))
        summed = _f(out + floor)
        lib.ndo_log_rn_array(_p(summed), summed.size, _p(out))
        lib.ndo_normalize_columns(_p(out), l0, mels)
        return l0, out

    # -- stem --
    def stem(self, feats):
        """StemOut rows [l3][dim] from the features [l0][mels]."""
        lib = O.lib()
        l0, mels, s = feats.shape[0], self.mels, self.stem_width
        l1 = (l0 + 1) // 2
        l2 = (l1 + 1) // 2
        l3 = (l2 + 1) // 2
        first = self.A("stem_first").reshape(9, s)
        stage0 = np.zeros((l1, 40, s), np.float32)
        for p in range(l1):
            o = np.zeros((40, s), np.float32)
            for dt in range(3):
                r = 2 * p - 1 + dt
                row = feats[r] if 0 <= r < l0 else np.zeros(mels, np.float32)
                for df in range(3):
                    freq = 2 * np.arange(40) - 1 + df
                    ok = (freq >= 0) & (freq < mels)
                    o[ok] = o[ok] + row[freq[ok]][:, None] * first[dt * 3 + df][None, :]
            lib.ndo_silu(_p(o), o.size)
            stage0[p] = o
        stage1 = self._stem_stage(stage0, l2, 40, 20, "stem_depthwise1", "stem_pointwise1")
        stage2 = self._stem_stage(stage1, l3, 20, 10, "stem_depthwise2", "stem_pointwise2")
        flat = _f(stage2.transpose(0, 2, 1).reshape(l3, s * 10))  # flat[c * 10 + f] = row[f * s + c]
        return self._mm("stem_out", O.prepare_cq(flat, 2))

    def _stem_stage(self, src, rows_out, freq_in, freq_out, depthwise, pointwise):
        """Depthwise 3x3 at stride 2 (Whistle.Depthwise, :326-344), the 2-bit
        pointwise matmul per (row, frequency) and SiLU."""
        s = self.stem_width
        w = self.A(depthwise).reshape(9, s)
        dw = np.zeros((rows_out, freq_out, s), np.float32)
        zero = np.zeros((freq_in, s), np.float32)
        for q in range(rows_out):
            rows = [src[2 * q - 1 + dt] if 0 <= 2 * q - 1 + dt < src.shape[0] else zero for dt in range(3)]
            o = np.zeros((freq_out, s), np.float32)
            for dt in range(3):
                for df in range(3):
                    freq = 2 * np.arange(freq_out) - 1 + df
                    ok = (freq >= 0) & (freq < freq_in)
                    o[ok] = o[ok] + rows[dt][freq[ok]] * w[dt * 3 + df][None, :]
            dw[q] = o
        y = self._mm(pointwise, O.prepare_cq(dw.reshape(rows_out * freq_out, s), 2))
        O.lib().ndo_silu(_p(y), y.size)
        return y.reshape(rows_out, freq_out, s)

    # -- encoder --
    def _zc(self, x, scale):
        out = np.zeros_like(x)
        O.lib().ndo_zero_centered_rms(_p(x), _p(scale), x.size, _p(out))
        return out

    def _mlp(self, prefix, pre_norm, residual):
        g = self.g
        host = [self.A(f"{prefix}.{n}") for n in MLP]
        ptrs = (ctypes.c_void_p * 13)(*[h.ctypes.data for h in host])
        pa = np.ascontiguousarray(self.perm("hyper.perm_a"), np.int32)
        pb = np.ascontiguousarray(self.perm("hyper.perm_b"), np.int32)
        for t in range(residual.shape[0]):
            O.lib().ndo_hadamard_mlp(ptrs, _p(pre_norm), _p(pa), _p(pb), self.dim, g["hada_rows"], g["hada_cols"], 0.5,
                                     _p(residual[t]))

    def encoder(self, stem_out):
        """RunEncoder (:794-828) and ExecuteEncoderFinal (:614-626): [frames][dim]."""
        g, lib = self.g, O.lib()
        F, d = stem_out.shape
        H, KV, QK, VD = g["heads"], g["kv_heads"], g["qk_dim"], g["v_dim"]
        width = LANES * d
        stream = np.repeat(_f(stem_out)[:, None, :], LANES, axis=1).copy()
        a_pre, b_pre = self.A("hyper.a_pre"), self.A("hyper.b_pre")
        a_post, b_post = self.A("hyper.a_post"), self.A("hyper.b_post")
        a_res, b_res = self.A("hyper.a_res"), self.A("hyper.b_res")
        cos_t, sin_t = np.zeros((F, QK // 2), np.float32), np.zeros((F, QK // 2), np.float32)
        lib.ndo_whistle_rope_tables(np.float32(g["rope_theta"]), QK, F, _p(cos_t), _p(sin_t))
        inv_sqrt = np.float32(1.0) / np.float32(np.sqrt(np.float32(QK)))
        sig = lambda v: np.float32(lib.ndo_sigmoid(float(v)))
        for l in range(self.encoder_layers):
            e = f"enc{l}."
            lane = l % LANES
            flat = stream.reshape(F, width)
            normalized = np.stack([flat[t] * np.float32(lib.ndo_inverse_rms(_p(_f(flat[t])), width))
                                   for t in range(F)])
            act = O.prepare_cq(normalized, 4)
            pre = self._mm("hyper.phi_pre", act, (l * LANES, l * LANES + LANES))
            post = self._mm("hyper.phi_post", act, (l * LANES, l * LANES + LANES))
            res = self._mm("hyper.phi_res", act, (l * 16, l * 16 + 16))
            u = np.zeros((F, d), np.float32)
            mix = np.zeros((F, 16), np.float32)
            post_gate = np.zeros((F, LANES), np.float32)
            for t in range(F):
                hpre = np.zeros(LANES, np.float32)
                for i in range(LANES):
                    zp = np.float32(np.float32(a_pre[l] * pre[t, i]) + b_pre[l * LANES + i]) + np.float32(
                        4.0 if i == lane else -4.0)
                    hpre[i] = sig(zp)
                    zq = np.float32(np.float32(a_post[l] * post[t, i]) + b_post[l * LANES + i]) + np.float32(
                        0.0 if i == lane else -4.0)
                    post_gate[t, i] = np.float32(2.0) * sig(zq)
                lib.ndo_mix4(_p(stream[t]), d, float(hpre[0]), float(hpre[1]), float(hpre[2]), float(hpre[3]),
                             _p(u[t]))
                logits = _f([np.float32(a_res[l] * res[t, i]) + b_res[l * 16 + i] for i in range(16)])
                mix[t] = O.sinkhorn4x4(logits)
            residual = u.copy()
            self._mlp(e + "mlp0", self.A(e + "pre_mlp_norm0"), residual)
            self._attention(e, residual, cos_t, sin_t, inv_sqrt)
            self._convolution(e, residual)
            self._mlp(e + "mlp", self.A(e + "pre_mlp_norm"), residual)
            nxt = np.zeros_like(stream)
            for t in range(F):
                lib.ndo_combine_diff4x4(_p(stream[t]), d, _p(mix[t]), _p(residual[t]), _p(u[t]), _p(post_gate[t]),
                                        _p(nxt[t]))
            stream = nxt
        final = self.A("final_norm")
        out = np.zeros((F, d), np.float32)
        for t in range(F):
            mean = np.zeros(d, np.float32)
            lib.ndo_mix4(_p(stream[t]), d, 0.25, 0.25, 0.25, 0.25, _p(mean))
            out[t] = self._zc(mean, final)
        return out

    def _attention(self, e, residual, cos_t, sin_t, inv_sqrt):
        """RunSelfAttention (:840-862): every frame attends every frame."""
        g, lib = self.g, O.lib()
        F, d = residual.shape
        H, KV, QK, VD = g["heads"], g["kv_heads"], g["qk_dim"], g["v_dim"]
        x = np.stack([self._zc(residual[t], self.A(e + "attn_norm")) for t in range(F)])
        act = O.prepare_cq(x, 2)
        q, k, v, gate = (self._mm(e + n, act) for n in ("q", "k", "v", "gate"))
        qn, kn = self.A(e + "q_norm"), self.A(e + "k_norm")
        q8, qs = np.zeros((F, H * QK), np.int8), np.zeros((F, H), np.float32)
        keys, ks = np.zeros((F, KV * QK), np.int8), np.zeros((F, KV), np.float32)
        vals, vs = np.zeros((F, KV * VD), np.int8), np.zeros((F, KV), np.float32)
        for t in range(F):
            qt, kt = _f(q[t]), _f(k[t])
            for h in range(H):
                qt[h * QK:(h + 1) * QK] = self._zc(_f(qt[h * QK:(h + 1) * QK]), qn)
            for h in range(KV):
                kt[h * QK:(h + 1) * QK] = self._zc(_f(kt[h * QK:(h + 1) * QK]), kn)
            lib.ndo_rope(_p(qt), H, QK, _p(cos_t[t]), _p(sin_t[t]))
            lib.ndo_rope(_p(kt), KV, QK, _p(cos_t[t]), _p(sin_t[t]))
            for h in range(H):
                q8[t, h * QK:(h + 1) * QK], qs[t, h] = O.quantize_int8(qt[h * QK:(h + 1) * QK])
            for h in range(KV):
                keys[t, h * QK:(h + 1) * QK], ks[t, h] = O.quantize_int8(kt[h * QK:(h + 1) * QK])
                vals[t, h * VD:(h + 1) * VD], vs[t, h] = O.quantize_int8(_f(v[t, h * VD:(h + 1) * VD]))
        out = np.zeros((F, H * VD), np.float32)
        group = H // KV
        for h in range(H):
            kvh = h // group
            kk = np.ascontiguousarray(keys[:, kvh * QK:(kvh + 1) * QK])
            vv = np.ascontiguousarray(vals[:, kvh * VD:(kvh + 1) * VD])
            kss, vss = np.ascontiguousarray(ks[:, kvh]), np.ascontiguousarray(vs[:, kvh])
            for t in range(F):
                out[t, h * VD:(h + 1) * VD] = O.attention_head(
                    np.ascontiguousarray(q8[t, h * QK:(h + 1) * QK]), float(qs[t, h]), kk, kss, vv, vss, QK, VD, 1, 0,
                    F - 1, QK, VD, float(inv_sqrt))
        gate = _f(gate)
        for t in range(F):
            lib.ndo_multiply_by_sigmoid(_p(out[t]), _p(gate[t]), H * VD)
        proj = self._mm(e + "out", O.prepare_cq(out, 2))
        post_norm = self.A(e + "post_attn_norm")
        attn_gate = float(lib.ndo_sigmoid(float(self.A(e + "attn_gate")[0])))
        for t in range(F):
            lib.ndo_post_norm_add(_p(residual[t]), _p(_f(proj[t])), _p(post_norm), attn_gate, d)

    def _convolution(self, e, residual):
        """RunConvolution (:864-876)."""
        lib = O.lib()
        F, d = residual.shape
        K = self.conv_kernel
        x = np.stack([self._zc(residual[t], self.A(e + "conv_norm")) for t in range(F)])
        glu = _f(self._mm(e + "pw1", O.prepare_cq(x, 2)))
        hidden = np.zeros((F, d), np.float32)
        for t in range(F):
            lib.ndo_glu(_p(_f(glu[t, :d])), _p(_f(glu[t, d:])), _p(hidden[t]), d)
        taps = self.A(e + "depthwise").reshape(K, d)
        out_norm = self.A(e + "conv_out_norm")
        rows = np.zeros((F, d), np.float32)
        for t in range(F):
            o = np.zeros(d, np.float32)
            for k in range(K):
                src = t + k - K // 2
                if 0 <= src < F:
                    o = o + taps[k] * hidden[src]
            r = self._zc(o, out_norm)
            lib.ndo_silu(_p(r), d)
            rows[t] = r
        proj = self._mm(e + "pw2", O.prepare_cq(rows, 2))
        residual += proj

    # -- the whole --
    def encode(self, pcm):
        """Whistle.Encode: the frame count; keeps mel, stem and encoder outputs."""
        l0, self.mel = self.features(pcm)
        if l0 == 0:
            self.stem_out = self.encoder_out = np.zeros((0, self.dim), np.float32)
            return 0
        self.stem_out = self.stem(self.mel)
        self.encoder_out = self.encoder(self.stem_out)
        return self.encoder_out.shape[0]

    def build_memory(self):
        """BuildCrossMemory: per decoder layer (keys int8 [frames][heads * qk],
        key scales [frames][heads], values int8 [frames][heads * vd], value
        scales [frames][heads])."""
        g, lib = self.g, O.lib()
        F, d = self.encoder_out.shape
        H, QK, VD = g["heads"], g["qk_dim"], g["v_dim"]
        half = d // 2
        sin_t, cos_t = np.zeros((F, half), np.float32), np.zeros((F, half), np.float32)
        lib.ndo_cross_position_tables(d, F, _p(sin_t), _p(cos_t))
        mix = np.float32(lib.ndo_sigmoid(float(self.A("position_mix")[0])))
        rows = self.encoder_out.copy()
        rows[:, :half] = rows[:, :half] + mix * sin_t
        rows[:, half:] = rows[:, half:] + mix * cos_t
        rows = _f(rows)
        for t in range(F):
            lib.ndo_fake_a8(_p(rows[t]), d)
        act = O.prepare_cq(rows, 2)
        memory = []
        for l in range(g["layers"]):
            kk = _f(self._mm(f"cross{l}.k", act))
            vv = _f(self._mm(f"cross{l}.v", act))
            kn = self.A(f"cross{l}.k_norm")
            keys, ks = np.zeros((F, H * QK), np.int8), np.zeros((F, H), np.float32)
            vals, vs = np.zeros((F, H * VD), np.int8), np.zeros((F, H), np.float32)
            for t in range(F):
                for h in range(H):
                    seg = self._zc(_f(kk[t, h * QK:(h + 1) * QK]), kn)
                    keys[t, h * QK:(h + 1) * QK], ks[t, h] = O.quantize_int8(seg)
                    vals[t, h * VD:(h + 1) * VD], vs[t, h] = O.quantize_int8(_f(vv[t, h * VD:(h + 1) * VD]))
            memory.append((keys, ks, vals, vs))
        return memory
