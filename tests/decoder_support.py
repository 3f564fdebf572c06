"""Helpers shared by the decoder parity tests: copy an engine's weights into
the CPU oracle and regenerate the synthetic prefix K/V on the host."""
import numpy as np

from attention_support import K_BYTE, K_OFF, KS_OFF, S_SLOT, V_BYTE, V_OFF, VS_OFF
from conftest import entry

KV_STREAM_SHIFT = 20


def oracle_decoder(oracle, engine):
    cfg = engine.model
    names = dict(oracle.LAYER_TENSORS)
    if getattr(cfg, "cross", 0):
        names.update(oracle.CROSS_TENSORS)
    layers = []
    for l in range(cfg.layers):
        layers.append({name: engine.read_tensor(name, dt, layer=l) for name, dt in names.items()})
    return oracle.Decoder(cfg, layers, engine.read_tensor("final_norm", np.float32),
                          engine.read_tensor("embedding", np.uint16), engine.read_tensor("w_head", np.int8),
                          engine.read_tensor("s_head", np.uint16), engine.capacity)


def prefix_kv(ops, oracle, decoder, kv, count, seed, session):
    """Fill positions [0, count) of an oracle KV dict the way
    ndl_slot_fill_synthetic does: fp16 normal from (seed, session) at index
    ((((layer*2 + kind) << 20) + pos) * heads + head) * 64 + d, quantized per
    (position, head) by the oracle's QuantizeInt8."""
    cfg = decoder.cfg
    H = cfg.heads
    for layer in range(cfg.layers):
        for kind, (vals, scales) in enumerate((("k", "ks"), ("v", "vs"))):
            first = ((layer * 2 + kind) << KV_STREAM_SHIFT) * H * 64
            raw = ops.synth_normal_f16(seed, session, count * H * 64, first=first)
            x = raw.view(np.float16).astype(np.float32).reshape(count * H, 64)
            q, s = oracle.quantize_rows(x)
            kv[vals][layer, :count] = q.reshape(count, H * 64)
            kv[scales][layer, :count] = s.reshape(count, H)


def read_slot_kv(engine, slot, positions):
    """Reads positions [0, positions) of a slot from the paged pool into the
    flat reference layout (k, v int8 [layers][positions][H*64]; ks, vs).
    Page record of (layer, head): K int8 in m16n8k32 A-fragment order
    (K_BYTE) with its scales at S_SLOT, then the V scales in position order
    and V dim-major (V_BYTE)."""
    cfg = engine.model
    H, L = cfg.heads, cfg.layers
    page_bytes = engine.page_bytes()
    n_pages = (positions + 63) // 64
    pages = [engine.slot_page(slot, i) for i in range(n_pages)]
    need = (max(pages) + 1) * page_bytes
    pool = engine.read_tensor("kv_pool", np.uint8, count=need)
    out = {"k": np.zeros((L, positions, H * 64), np.int8), "v": np.zeros((L, positions, H * 64), np.int8),
           "ks": np.zeros((L, positions, H), np.float32), "vs": np.zeros((L, positions, H), np.float32)}
    for pi, page in enumerate(pages):
        lo, hi = pi * 64, min(positions, pi * 64 + 64)
        n = hi - lo
        for l in range(L):
            for h in range(H):
                blk = pool[page * page_bytes + (l * H + h) * 8704:][:8704]
                out["k"][l, lo:hi, h * 64:(h + 1) * 64] = blk[K_OFF:K_OFF + 4096][K_BYTE[:n]].view(np.int8)
                out["ks"][l, lo:hi, h] = blk[KS_OFF:KS_OFF + 256].view(np.float32)[S_SLOT[:n]]
                out["vs"][l, lo:hi, h] = blk[VS_OFF:VS_OFF + 256].view(np.float32)[:n]
                out["v"][l, lo:hi, h * 64:(h + 1) * 64] = blk[V_OFF:V_OFF + 4096][V_BYTE[:n]].view(np.int8)
    return out


def top2_margin(x):
    s = np.sort(x)
    return float(s[-1] - s[-2])


def parallel_map(fn, items, threads=None):
    """fn over items on a thread pool (the oracle's ctypes calls release the
    GIL, so sessions run on all host cores); results in item order."""
    import os
    from concurrent.futures import ThreadPoolExecutor

    with ThreadPoolExecutor(max_workers=threads or os.cpu_count() or 1) as pool:
        return list(pool.map(fn, items))


def oracle_greedy(ops, oracle, dec, seed, session, length, token, steps):
    """One session's greedy chain on the oracle: prefix K/V of `length`
    positions from (seed, session), then `steps` rows starting with `token`
    at position `length`, each next token the first maximum of the logits
    (Ops.ArgMax).  Returns (ids [steps], logits [steps][vocab])."""
    kv = dec.new_kv()
    prefix_kv(ops, oracle, dec, kv, length, seed, session)
    ids, logits = [], []
    pos = length
    for _ in range(steps):
        lg = dec.row(int(token), pos, kv)
        logits.append(lg)
        token = int(np.argmax(lg))
        ids.append(token)
        pos += 1
    return ids, logits


def oracle_request(oracle, dec, prompt, max_new, mask, vocab, stop=-1):
    """One request on the oracle, as a session serves it alone: the prompt
    one row at a time from an empty cache, then greedy decoding with the
    request's vocabulary mask (Ops.ArgMaxMasked; plain argmax without a
    mask) until max_new tokens, the stop token or an empty mask."""
    kv = dec.new_kv()
    pos = 0
    for t in prompt:
        logits = dec.row(int(t), pos, kv)
        pos += 1
    out = []
    while True:
        tok = oracle.argmax_masked(logits, mask, vocab) if mask is not None else int(np.argmax(logits))
        if tok < 0:
            break
        out.append(int(tok))
        if len(out) >= max_new or tok == stop:
            break
        logits = dec.row(int(tok), pos, kv)
        pos += 1
    return out
