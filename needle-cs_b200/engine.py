"""Host-side mirror of the reference's BatchedEngine over the C ABI.

Method names and argument meaning follow src/Needle/BatchEngine.cs:5-50
(Slots, Capacity, VocabSize, SlotLength, ResetSlot, MarkSlot, RewindSlot,
FeedSlot, ForwardBatch, BatchLogitsRow).  Errors raise NeedleError with the
ABI status: ContextExhausted (3) where the reference throws
InvalidOperationException("context capacity exceeded"), invalid argument
(100) where it throws ArgumentOutOfRangeException.
"""
import ctypes
from dataclasses import dataclass

import numpy as np

from ._native import PROF_CLASSES, DecoderConfig, EngineConfig, call, lib


@dataclass
class SyntheticDecoder:
    """The synthetic Needle-3-shaped decoder of the benchmark configs."""
    layers: int = 12
    dim: int = 512
    heads: int = 8
    head_dim: int = 64
    ffn: int = 2048
    vocab: int = 8192
    rope_theta: float = 10000.0
    seed: int = 1
    cross: int = 0  # 1: a cross-attention block per layer (Whistle-shaped decoder)

    def native(self):
        return DecoderConfig(self.layers, self.dim, self.heads, self.head_dim, self.ffn, self.vocab, self.rope_theta,
                             self.seed, int(self.cross))


def whistle_decoder(seed=3):
    """The cfg4 decoder: 4 layers, d 384, 6x64 heads, SwiGLU 1536, vocab 51865,
    cross-attention to a per-utterance encoder memory."""
    return SyntheticDecoder(layers=4, dim=384, heads=6, head_dim=64, ffn=1536, vocab=51865, seed=seed, cross=1)


def _i32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


class BatchedEngine:
    def __init__(self, model=None, slots=8, context_length=1024, chunk_size=64, device=0, max_heads=None,
                 kv_pages=0):
        self.model = model or SyntheticDecoder()
        self.chunk = chunk_size
        max_heads = max_heads or chunk_size
        cfg = EngineConfig(device, slots, context_length, kv_pages, chunk_size, max_heads)
        handle = ctypes.c_void_p()
        mc = self.model.native()
        call("ndl_engine_create", ctypes.byref(cfg), ctypes.byref(mc), ctypes.byref(handle))
        self._h = handle
        self.slots = slots
        self.capacity = context_length
        self.vocab_size = self.model.vocab
        self.max_heads = max_heads
        self._last_heads = 0

    @classmethod
    def from_model(cls, model, slots=8, context_length=512, chunk_size=64, max_heads=None):
        """A batched engine over a loaded Needle-3 archive (needle_cs_b200.model.Model
        on a device): ndl_engine_create_model.  Forwards run the model's
        RunLayerBatch chain; the model must outlive the engine."""
        self = cls.__new__(cls)
        self.model = model
        self.chunk = chunk_size
        max_heads = max_heads or chunk_size
        info = model.info
        cfg = EngineConfig(info["device"], slots, context_length, 0, chunk_size, max_heads)
        handle = ctypes.c_void_p()
        call("ndl_engine_create_model", ctypes.byref(cfg), model._h, ctypes.byref(handle))
        self._h = handle
        self.slots = slots
        self.capacity = context_length
        self.vocab_size = info["vocab"]
        self.max_heads = max_heads
        self._last_heads = 0
        return self

    # -- lifetime --
    def close(self):
        if self._h:
            lib().ndl_engine_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def stream(self):
        s = ctypes.c_void_p()
        call("ndl_engine_stream", self._h, ctypes.byref(s))
        return s.value

    # -- slots (BatchEngine.cs:23-30) --
    def slot_length(self, slot):
        n = ctypes.c_int()
        call("ndl_slot_length", self._h, slot, ctypes.byref(n))
        return n.value

    def reset_slot(self, slot):
        call("ndl_slot_reset", self._h, slot)

    def mark_slot(self, slot):
        call("ndl_slot_mark", self._h, slot)

    def rewind_slot(self, slot):
        call("ndl_slot_rewind", self._h, slot)

    def slot_page(self, slot, index):
        p = ctypes.c_int()
        call("ndl_slot_page", self._h, slot, index, ctypes.byref(p))
        return p.value

    def fill_synthetic(self, slot, count, seed, session):
        call("ndl_slot_fill_synthetic", self._h, slot, count, seed, session)

    # -- steps --
    def forward_batch(self, tokens, row_slots, head_rows=()):
        """EngineCore.ForwardBatch (Engine.cs:2303-2350)."""
        t, s, h = _i32(tokens), _i32(row_slots), _i32(head_rows)
        if t.size != s.size:
            raise ValueError("one slot per token")
        call("ndl_forward_batch", self._h, t.ctypes.data, s.ctypes.data, t.size, h.ctypes.data if h.size else None,
             h.size)
        self._last_heads = h.size

    def feed_slot(self, slot, tokens, compute_logits=True):
        """BatchedEngine.FeedSlot / EngineCore.FeedSlot (Engine.cs:2285-2301): chunks of `chunk` rows."""
        tokens = _i32(tokens)
        if self.slot_length(slot) + tokens.size > self.capacity:
            from ._native import NeedleError

            raise NeedleError(3, "context capacity exceeded")
        for start in range(0, tokens.size, self.chunk):
            part = tokens[start:start + self.chunk]
            last = start + part.size == tokens.size
            heads = [part.size - 1] if (last and compute_logits) else []
            self.forward_batch(part, [slot] * part.size, heads)

    def batch_logits_row(self, compact_row):
        out = np.empty(self.vocab_size, np.float32)
        call("ndl_batch_logits_row", self._h, compact_row, out.ctypes.data)
        return out

    def sample_argmax(self, masks=None, with_probs=False):
        n = self._last_heads
        ids = np.empty(n, np.int32)
        probs = np.empty(n, np.float32) if with_probs else None
        if masks is not None:
            masks = np.ascontiguousarray(masks, dtype=np.uint32).reshape(n, -1)
            call("ndl_sample_argmax", self._h, masks.ctypes.data, masks.shape[1], ids.ctypes.data,
                 probs.ctypes.data if with_probs else None)
        else:
            call("ndl_sample_argmax", self._h, None, 0, ids.ctypes.data, probs.ctypes.data if with_probs else None)
        return (ids, probs) if with_probs else ids

    # -- cross memory (Whistle-shaped decoders) --
    def set_memory(self, slot, memory_f16_bits):
        """Projects fp16 memory [frames][dim] (uint16 bits) into the K/V pages of an empty slot."""
        m = np.ascontiguousarray(memory_f16_bits, dtype=np.uint16)
        call("ndl_slot_set_memory", self._h, slot, m.ctypes.data, m.shape[0])

    def fill_memory_synthetic(self, slot, frames, seed, utterance):
        call("ndl_slot_fill_memory_synthetic", self._h, slot, frames, seed, utterance)

    def attach_memory(self, slot, memory_slot):
        call("ndl_slot_attach_memory", self._h, slot, memory_slot)

    def copy_slot(self, dst, src):
        """Engine.CopyFrom (Engine.cs:367-379): dst becomes a copy of src."""
        call("ndl_slot_copy", self._h, dst, src)

    # -- primed prefixes (Engine.cs:398-464) and prefix sharing --
    def prefix_bytes(self, slot):
        """Engine.PrimedPrefixBytes: bytes of the slot's marked-prefix blob."""
        n = ctypes.c_size_t()
        call("ndl_slot_prefix_bytes", self._h, slot, ctypes.byref(n))
        return n.value

    def export_prefix(self, slot):
        """Engine.ExportPrimedPrefix: the slot's marked prefix as a blob (bytes)."""
        buf = np.empty(self.prefix_bytes(slot), np.uint8)
        call("ndl_slot_export_prefix", self._h, slot, buf.ctypes.data, buf.size)
        return buf.tobytes()

    def import_prefix(self, slot, blob):
        """Engine.ImportPrimedPrefix: the slot's cache becomes the blob's prefix."""
        b = np.frombuffer(blob, np.uint8)
        call("ndl_slot_import_prefix", self._h, slot, b.ctypes.data, b.size)

    def share_prefix(self, dst, src):
        """dst takes src's marked prefix by reference (shared pages, copy on write)."""
        call("ndl_slot_share_prefix", self._h, dst, src)

    def time_attention(self, layer=0, reps=10):
        """Average ms of the last step's self-attention launch of `layer`, timed alone."""
        ms = ctypes.c_float()
        call("ndl_engine_time_attention", self._h, layer, reps, ctypes.byref(ms))
        return ms.value

    def free_pages(self):
        n = ctypes.c_int()
        call("ndl_engine_free_pages", self._h, ctypes.byref(n))
        return n.value

    def set_mask(self, slot, mask=None):
        """Keeps a vocabulary bitmask for `slot` on the device (None clears it)."""
        if mask is None:
            call("ndl_engine_set_mask", self._h, slot, None, 0)
            return
        m = np.ascontiguousarray(mask, dtype=np.uint32)
        call("ndl_engine_set_mask", self._h, slot, m.ctypes.data, m.size)

    def sample_argmax_slots(self, slots, with_probs=False):
        """ArgMaxMasked of every head row with the stored mask of slots[h]."""
        n = self._last_heads
        sl = _i32(slots)
        assert sl.size == n, (sl.size, n)
        ids = np.empty(n, np.int32)
        probs = np.empty(n, np.float32) if with_probs else None
        call("ndl_sample_argmax_slots", self._h, sl.ctypes.data, ids.ctypes.data,
             probs.ctypes.data if with_probs else None)
        return (ids, probs) if with_probs else ids

    def logits_sparse(self, rows, id_lists, values=True, pick=False, with_probs=False):
        """Engine.LogitsForBatchRow for several requests: the logits of batch
        row rows[r] of the last step at the vocabulary ids id_lists[r]; with
        pick, ArgMaxSparse's id per request (and BestProbability with
        with_probs).  Returns (values per request, picks, probs), absent parts
        None."""
        rw = _i32(rows)
        lists = [_i32(x) for x in id_lists]
        assert len(lists) == rw.size, (len(lists), rw.size)
        offsets = np.zeros(rw.size + 1, np.int32)
        offsets[1:] = np.cumsum([x.size for x in lists])
        flat = np.concatenate(lists) if lists else np.zeros(0, np.int32)
        flat = np.ascontiguousarray(flat, np.int32)
        total = int(offsets[-1])
        vals = np.empty(max(total, 1), np.float32) if values else None
        picks = np.empty(max(rw.size, 1), np.int32) if (pick or with_probs) else None
        probs = np.empty(max(rw.size, 1), np.float32) if with_probs else None
        call("ndl_logits_sparse", self._h, rw.size, rw.ctypes.data, offsets.ctypes.data,
             flat.ctypes.data if total else None, vals.ctypes.data if values else None,
             picks.ctypes.data if picks is not None else None, probs.ctypes.data if with_probs else None)
        per = [vals[offsets[r]:offsets[r + 1]].copy() for r in range(rw.size)] if values else None
        return per, (picks[:rw.size] if picks is not None else None), (probs[:rw.size] if with_probs else None)

    def sample_topk(self, k, mask_special_023=False, with_probs=False):
        n = self._last_heads
        ids = np.empty((n, k), np.int32)
        lp = np.empty((n, k), np.float32)
        pr = np.empty((n, k), np.float32) if with_probs else None
        call("ndl_sample_topk", self._h, k, int(mask_special_023), ids.ctypes.data, lp.ctypes.data,
             pr.ctypes.data if with_probs else None)
        return ids, lp, pr

    def use_graphs(self, enable=True):
        call("ndl_engine_use_graphs", self._h, int(enable))

    def use_pdl(self, enable=True):
        call("ndl_engine_use_pdl", self._h, int(enable))

    def profile(self, enable=True):
        call("ndl_engine_profile", self._h, int(enable))

    def profile_read(self, reset=True):
        """{class: (ms, launches)} accumulated since the last reset."""
        ms = np.zeros(len(PROF_CLASSES), np.float64)
        n = np.zeros(len(PROF_CLASSES), np.int64)
        call("ndl_engine_profile_read", self._h, ms.ctypes.data, n.ctypes.data, int(reset))
        return {c: (float(ms[i]), int(n[i])) for i, c in enumerate(PROF_CLASSES)}

    def sync(self):
        call("ndl_engine_sync", self._h)

    # -- export --
    def tensor_bytes(self, name, layer=-1):
        p = ctypes.c_void_p()
        n = ctypes.c_size_t()
        call("ndl_engine_tensor", self._h, name.encode(), layer, ctypes.byref(p), ctypes.byref(n))
        return p.value, n.value

    def read_tensor(self, name, dtype, layer=-1, count=None):
        _, nbytes = self.tensor_bytes(name, layer)
        itemsize = np.dtype(dtype).itemsize
        count = nbytes // itemsize if count is None else count
        out = np.empty(count, dtype)
        call("ndl_engine_read_tensor", self._h, name.encode(), layer, out.ctypes.data, count * itemsize)
        return out

    def page_bytes(self):
        n = ctypes.c_size_t()
        call("ndl_engine_page_bytes", self._h, ctypes.byref(n))
        return n.value
