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
