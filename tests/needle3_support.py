"""The CPU oracle of the Needle-3 decode step over an archive written by
cact_support.needle3_decoder_archive (host tensors from the loader and the
archive's CQ records)."""
import numpy as np


def oracle_for(archive, model, slots, capacity):
    from oracle.needle3 import Needle3Oracle

    rec = {(r[0], r[1]): r[6] for r in archive.records}

    def cq(role, index):
        _, codes, norms, rows, cols, bits = rec[(role, index)]
        return codes.reshape(rows, -1), norms.reshape(rows, -1), rows, cols, bits

    cache = {}

    def dense(role, index=0):
        key = (role, index)
        if key not in cache:
            cache[key] = np.ascontiguousarray(model.host(role, index), np.float32)
        return cache[key]

    def perm(role):
        return np.ascontiguousarray(model.host(role, 0), np.int32)

    return Needle3Oracle(model.info, archive.levels, dense, cq, perm, slots, capacity)


def oracle_from_archive(archive, slots, capacity):
    """The same oracle built from the archive writer's records alone (no
    library): dense fp16 tensors by Scalar.HalfToSingle, the geometry as the
    loader derives it."""
    from cact_support import half_to_single
    from oracle.needle3 import Needle3Oracle

    g = archive.g
    rec = {(r[0], r[1]): r[6] for r in archive.records}
    rows = 1 << ((g["hada_n"] - 1).bit_length() // 2)
    info = dict(g, hada_rows=rows, hada_cols=g["hada_n"] // rows, order_count=len(g["orders"]),
                site_count=len(g["sites"]), vocab=g["vocab"])

    def cq(role, index):
        _, codes, norms, nrows, cols, bits = rec[(role, index)]
        return codes.reshape(nrows, -1), norms.reshape(nrows, -1), nrows, cols, bits

    def dense(role, index=0):
        kind, v = rec[(role, index)][:2]
        return half_to_single(v, exact=True) if kind == "dense16" else np.ascontiguousarray(v, np.float32)

    def perm(role):
        return np.ascontiguousarray(rec[(role, 0)][1], np.int32)

    return Needle3Oracle(info, archive.levels, dense, cq, perm, slots, capacity)
