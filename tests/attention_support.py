"""Builds paged KV pools in the library's page layout from natural-layout
K/V, for the standalone attention tests."""
import numpy as np

PAGE_POS = 64
BLOCK = 8704


def k_slot(d):
    """Storage byte of query dim d (the B-fragment order of both k-steps)."""
    return ((d & 15) >> 2) * 16 + (d >> 4) * 4 + (d & 3)


def frag_byte(row, col):
    """Byte of (row, col) of a 64x64 int8 matrix in m16n8k32 A-fragment order."""
    return ((row >> 4) * 1024 + (col >> 5) * 512 + ((row & 7) * 4 + ((col >> 2) & 3)) * 16
            + (((row >> 3) & 1) + 2 * ((col >> 4) & 1)) * 4 + (col & 3))


def scale_slot(p):
    """Index of position p's K scale (the lane order of the QK results)."""
    return 2 * ((p & 7) * 4 + ((p >> 4) & 3)) + ((p >> 3) & 1)


def v_byte(p, d):
    """Byte of (position p, dim d) within a page's V matrix: dim-major, the
    four 16-byte position chunks of dim d rotated by (d >> 1) & 3."""
    return d * 64 + ((((p >> 4) ^ ((d >> 1) & 3)) << 4) | (p & 15))


# a (layer, head) record: K half [K 0:4096][K scales 4096:4352], V half [V scales 4352:4608][V 4608:8704]
K_OFF, KS_OFF, VS_OFF, V_OFF = 0, 4096, 4352, 4608
K_ORDER = np.array([k_slot(d) for d in range(64)])
K_BYTE = np.array([[frag_byte(p, d) for d in range(64)] for p in range(64)])  # [position][dim] -> byte
V_BYTE = np.array([[v_byte(p, d) for d in range(64)] for p in range(64)])  # within the V matrix
S_SLOT = np.array([scale_slot(p) for p in range(64)])  # K scales


def make_case(seed, lengths, heads, layers=2, layer=1, max_pages=17):
    """Random natural-layout K/V/q and the matching paged pool.  Slot s owns
    pages s*max_pages .. ; returns a dict of numpy arrays."""
    rng = np.random.default_rng(seed)
    rows = len(lengths)
    page_bytes = layers * heads * BLOCK
    pool = np.zeros(rows * max_pages * page_bytes, np.uint8)
    cap = max_pages * PAGE_POS
    K = rng.integers(-128, 128, (rows, cap, heads, 64), dtype=np.int8)
    V = rng.integers(-128, 128, (rows, cap, heads, 64), dtype=np.int8)
    KS = rng.uniform(0.0005, 0.004, (rows, cap, heads)).astype(np.float32)
    VS = rng.uniform(0.001, 0.05, (rows, cap, heads)).astype(np.float32)
    Q = rng.integers(-128, 128, (rows, heads, 64), dtype=np.int8)
    QS = rng.uniform(0.2, 0.8, (rows, heads)).astype(np.float32)
    for s, n in enumerate(lengths):
        for pg in range((n + 63) // 64):
            page = s * max_pages + pg
            lo, hi = pg * 64, min(n, pg * 64 + 64)
            cnt = hi - lo
            for h in range(heads):
                base = page * page_bytes + (layer * heads + h) * BLOCK
                blk = pool[base:base + BLOCK]
                kr = np.zeros(4096, np.uint8)
                kr[K_BYTE[:cnt]] = K[s, lo:hi, h].view(np.uint8)
                blk[K_OFF:K_OFF + 4096] = kr
                ks = np.zeros(64, np.float32)
                ks[S_SLOT[:cnt]] = KS[s, lo:hi, h]
                blk[KS_OFF:KS_OFF + 256] = ks.view(np.uint8)
                vs = np.zeros(64, np.float32)
                vs[:cnt] = VS[s, lo:hi, h]
                blk[VS_OFF:VS_OFF + 256] = vs.view(np.uint8)
                vm = np.zeros(4096, np.uint8)
                vm[V_BYTE[:cnt]] = V[s, lo:hi, h].view(np.uint8)
                blk[V_OFF:V_OFF + 4096] = vm
    q_perm = np.zeros((rows, heads, 64), np.int8)
    q_perm[:, :, K_ORDER] = Q
    page_table = np.array([[s * max_pages + i for i in range(max_pages)] for s in range(rows)], np.int32)
    return dict(pool=pool, page_bytes=page_bytes, K=K, V=V, KS=KS, VS=VS, Q=Q, QS=QS, q_perm=q_perm,
                page_table=page_table, row_slot=np.arange(rows, dtype=np.int32),
                row_pos=np.array([n - 1 for n in lengths], np.int32), heads=heads, layer=layer)


def oracle_out(oracle, case, lengths, tier="simd"):
    """The oracle's attention of every (row, head): the reference's AVX2 tier
    (Attention.GroupAvx2, which the CUDA kernel follows bit for bit) or its
    scalar tier (Scalar.AttentionHead)."""
    rows, heads = len(lengths), case["heads"]
    out = np.zeros((rows, heads, 64), np.float32)
    for r, n in enumerate(lengths):
        for h in range(heads):
            keys = np.ascontiguousarray(case["K"][r, :n, h])
            vals = np.ascontiguousarray(case["V"][r, :n, h])
            fn = oracle.attention_head_simd if tier == "simd" else oracle.attention_head
            out[r, h] = fn(case["Q"][r, h], np.float32(case["QS"][r, h]), keys,
                           np.ascontiguousarray(case["KS"][r, :n, h]), vals,
                           np.ascontiguousarray(case["VS"][r, :n, h]), 64, 64, 1, 0, n - 1, 64, 64,
                           np.float32(0.125))
    return out
