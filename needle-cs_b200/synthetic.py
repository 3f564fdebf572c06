"""Host-side generation of the synthetic decoder and its prefix KV.

The same tensors the engine generates on the device (ndl_engine_create,
ndl_slot_fill_synthetic), built on the host with the library's host
generators, for CPU baselines and for checking the device generation.

Stream ids under the model seed: embedding 1, final norm 2, layer l field f
at 100 + 16*l + f with f = 0 w_qkv, 1 s_qkv, 2 w_o, 3 s_o, 4 w_gu, 5 s_gu,
6 w_d, 7 s_d, 8 attn_norm, 9 ffn_norm.  Weights are U{-127..127} int8,
scales fp16 U(0.001, 0.02), norms 1 + 0.1*normal (fp32), the embedding fp16
0.02*normal, and the head int8 quantized from the embedding per
(row, 32-group) with s = fp16(max|e|/127), w = clamp(rint(e/float(s)), +-127).
Cross-attention blocks (decoders with `cross`): layer l field f at
5000 + 16*l + f with f = 0 w_cq, 1 s_cq, 2 w_ckv, 3 s_ckv, 4 w_co, 5 s_co,
6 cross_norm; an utterance's encoder memory is fp16 N(0,1) [frames][dim]
under stream 2^40 + utterance.
"""
import numpy as np

from . import ops

FIELDS = ["w_qkv", "s_qkv", "w_o", "s_o", "w_gu", "s_gu", "w_d", "s_d", "attn_norm", "ffn_norm"]
CROSS_FIELDS = ["w_cq", "s_cq", "w_ckv", "s_ckv", "w_co", "s_co", "cross_norm"]
MEMORY_STREAM = 1 << 40
KV_STREAM_SHIFT = 20


def _norm(seed, stream, n):
    z = ops.synth_normal_f32(seed, stream, n)
    return (np.float32(1.0) + np.float32(0.1) * z).astype(np.float32)


def quantize_head(embedding_bits, vocab, dim):
    e = embedding_bits.view(np.float16).astype(np.float32).reshape(vocab, dim // 32, 32)
    peak = np.abs(e).max(axis=2)
    s16 = np.where(peak > 0, peak / np.float32(127.0), np.float32(1.0)).astype(np.float32).astype(np.float16)
    sf = s16.astype(np.float32)
    inv = (np.float32(1.0) / sf).astype(np.float32)
    w = np.clip(np.rint(e * inv[:, :, None]), -127, 127).astype(np.int8)
    return w.reshape(vocab, dim), s16.view(np.uint16).reshape(vocab, dim // 32)


def decoder_weights(cfg):
    """Returns (layers: list of dicts, final_norm, embedding_bits, w_head, s_head)."""
    seed, d, F, V = cfg.seed, cfg.dim, cfg.ffn, cfg.vocab
    G, GF = d // 32, F // 32
    shapes = {"w_qkv": (3 * d * d, "i8"), "s_qkv": (3 * d * G, "s"), "w_o": (d * d, "i8"), "s_o": (d * G, "s"),
              "w_gu": (2 * F * d, "i8"), "s_gu": (2 * F * G, "s"), "w_d": (d * F, "i8"), "s_d": (d * GF, "s"),
              "attn_norm": (d, "n"), "ffn_norm": (d, "n"),
              "w_cq": (d * d, "i8"), "s_cq": (d * G, "s"), "w_ckv": (2 * d * d, "i8"), "s_ckv": (2 * d * G, "s"),
              "w_co": (d * d, "i8"), "s_co": (d * G, "s"), "cross_norm": (d, "n")}

    def gen(name, stream):
        count, kind = shapes[name]
        if kind == "i8":
            return ops.synth_int8(seed, stream, count)
        if kind == "s":
            return ops.synth_uniform_f16(seed, stream, count, 0.001, 0.02)
        return _norm(seed, stream, count)

    layers = []
    for l in range(cfg.layers):
        t = {name: gen(name, 100 + 16 * l + f) for f, name in enumerate(FIELDS)}
        if getattr(cfg, "cross", 0):
            t.update({name: gen(name, 5000 + 16 * l + f) for f, name in enumerate(CROSS_FIELDS)})
        layers.append(t)
    final_norm = _norm(seed, 2, d)
    emb = ops.synth_normal_f16(seed, 1, V * d, scale=0.02)
    w_head, s_head = quantize_head(emb, V, d)
    return layers, final_norm, emb, w_head.reshape(-1), s_head.reshape(-1)


def prefix_kv_values(seed, session, layer, kind, count, heads):
    """fp16 prefix K (kind 0) or V (kind 1) of one session and layer as
    float32 [count][heads][64]."""
    first = ((layer * 2 + kind) << KV_STREAM_SHIFT) * heads * 64
    raw = ops.synth_normal_f16(seed, session, count * heads * 64, first=first)
    return raw.view(np.float16).astype(np.float32).reshape(count, heads, 64)


def memory_values(seed, utterance, frames, dim):
    """fp16 N(0,1) encoder memory of one utterance as float32 [frames][dim]."""
    raw = ops.synth_normal_f16(seed, MEMORY_STREAM + utterance, frames * dim)
    return raw.view(np.float16).astype(np.float32).reshape(frames, dim)
