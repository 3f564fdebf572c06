"""Needle-3 model archives (.cact): the mirror of the reference's
Model.FromBytes / Model.Open (src/Needle/Model.cs:307-404) over
ndl_model_load.

A malformed archive raises InvalidDataError (the reference's
InvalidDataException); an unsupported geometry raises NotSupportedError
(NotSupportedException).  The messages are the reference's.  Tensors are
named by role and index (layer, site or probe head), e.g.
``model.tensor("layer.q", 3)``.  After an upload (device >= 0), a tensor's
device addresses feed the CQ and Needle-3 entry points directly.
"""
import ctypes

import numpy as np

from ._native import NeedleError, call, lib

MALFORMED = 107  # NDL_ERR_MALFORMED_MODEL
UNSUPPORTED = 105  # NDL_ERR_UNSUPPORTED

DENSE, CQ, PERMUTATION, CQ_ROWS, RAW = range(5)


class InvalidDataError(NeedleError, ValueError):
    """The archive is not a well-formed .cact file."""


class NotSupportedError(NeedleError):
    """The archive is well formed but its geometry is not supported."""


class Codebook(ctypes.Structure):
    _fields_ = [("levels", ctypes.c_float * 16), ("bytes", ctypes.c_uint8 * 32), ("byte_scale", ctypes.c_float)]


class ModelInfo(ctypes.Structure):
    _fields_ = [("magic", ctypes.c_uint32), ("tensors", ctypes.c_int), ("codebook_entries", ctypes.c_int),
                ("length", ctypes.c_int64), ("tokenizer_bytes", ctypes.c_int64),
                ("has_audio", ctypes.c_int), ("has_confidence", ctypes.c_int), ("has_embedding_head", ctypes.c_int),
                ("probe_heads", ctypes.c_int), ("confidence_head", ctypes.c_int), ("embedding_head", ctypes.c_int),
                ("probe_codes", ctypes.c_int * 16)] + [
                   (n, ctypes.c_int) for n in (
                       "vocab", "dim", "heads", "kv_heads", "layers", "qk_dim", "v_dim", "max_seq", "hada_n", "lanes",
                       "sliding_window", "conv_taps", "engram_slots", "engram_sub", "engram_tables",
                       "engram_conv_taps", "engram_dilation", "engram_seed_heads", "kv_window",
                       "order_count", "site_count")] + [
                ("global_mask", ctypes.c_uint64), ("rope_theta", ctypes.c_float),
                ("orders", ctypes.c_int * 4), ("sites", ctypes.c_int * 16),
                ("hada_rows", ctypes.c_int), ("hada_cols", ctypes.c_int),
                ("device", ctypes.c_int), ("device_bytes", ctypes.c_size_t)]

    def as_dict(self):
        out = {}
        for name, _ in self._fields_:
            v = getattr(self, name)
            out[name] = list(v) if isinstance(v, ctypes.Array) else v
        out["orders"] = out["orders"][:self.order_count]
        out["sites"] = out["sites"][:self.site_count]
        out["probe_codes"] = out["probe_codes"][:self.probe_heads]
        return out


class Tensor(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int), ("record", ctypes.c_int), ("dtype", ctypes.c_int), ("ndim", ctypes.c_int),
                ("shape", ctypes.c_int64 * 4), ("offset", ctypes.c_uint64), ("bytes", ctypes.c_uint64),
                ("count", ctypes.c_int64), ("rows", ctypes.c_int), ("cols", ctypes.c_int), ("bits", ctypes.c_int),
                ("values", ctypes.c_void_p), ("permutation", ctypes.c_void_p), ("indices", ctypes.c_void_p),
                ("norms", ctypes.c_void_p), ("book", ctypes.POINTER(Codebook))]


def _raise_typed(err):
    if err.status == MALFORMED:
        raise InvalidDataError(err.status, str(err).split(": ", 1)[1]) from None
    if err.status == UNSUPPORTED:
        raise NotSupportedError(err.status, str(err).split(": ", 1)[1]) from None
    raise err


class Model:
    """A loaded archive (Model.FromBytes); ``device`` None or < 0: host only."""

    def __init__(self, data, device=None):
        buf = np.frombuffer(bytes(data), np.uint8) if not isinstance(data, np.ndarray) else data.view(np.uint8)
        handle = ctypes.c_void_p()
        try:
            call("ndl_model_load", buf.ctypes.data if buf.size else None, buf.size,
                 -1 if device is None else int(device), ctypes.byref(handle))
        except NeedleError as err:
            _raise_typed(err)
        self._h = handle

    @classmethod
    def from_bytes(cls, data, device=None):
        return cls(data, device)

    @classmethod
    def open(cls, path, device=None):
        """Model.Open: a missing file raises FileNotFoundError."""
        with open(path, "rb") as f:
            return cls(f.read(), device)

    @property
    def info(self):
        info = ModelInfo()
        call("ndl_model_get_info", self._h, ctypes.byref(info))
        return info.as_dict()

    @property
    def layer_count(self):
        return self.info["layers"]

    @property
    def vocab_size(self):
        return self.info["vocab"]

    def tensors(self):
        """[(role, index)] in the archive's record order."""
        n = ctypes.c_int()
        call("ndl_model_tensor_count", self._h, ctypes.byref(n))
        out = []
        for i in range(n.value):
            role, index = ctypes.c_char_p(), ctypes.c_int()
            call("ndl_model_tensor_name", self._h, i, ctypes.byref(role), ctypes.byref(index))
            out.append((role.value.decode(), index.value))
        return out

    def tensor(self, role, index=0):
        t = Tensor()
        call("ndl_model_get_tensor", self._h, role.encode(), index, ctypes.byref(t))
        return t

    def host(self, role, index=0):
        """The host copy of a dense (float32) or permutation (int32) tensor."""
        t = self.tensor(role, index)
        out = np.empty(t.count, np.float32 if t.kind == DENSE else np.int32)
        call("ndl_model_read_host", self._h, role.encode(), index, out.ctypes.data, out.nbytes)
        return out

    def tokenizer_blob(self):
        blob, n = ctypes.c_void_p(), ctypes.c_size_t()
        call("ndl_model_tokenizer", self._h, ctypes.byref(blob), ctypes.byref(n))
        return ctypes.string_at(blob, n.value) if n.value else b""

    # -- blocks on the uploaded weights (torch CUDA tensors, contiguous) --
    def engram_workspace_bytes(self, count):
        return int(lib().ndl_engram_workspace(self._h, count))

    def apply_engram(self, site, tokens, row_slots, slot_length, slot_prev, history_in, history_out, x, residual,
                     workspace=None):
        """ApplyEngramBatch for one site on torch's current stream: residual
        [count][dim] updated, history_out [slots][9][dim] gets the batch
        slots' new histories (ndl_engram_apply)."""
        import torch

        count = int(row_slots.numel())
        if workspace is None:
            workspace = torch.empty(self.engram_workspace_bytes(count), dtype=torch.uint8, device=residual.device)
        call("ndl_engram_apply", self._h, site, tokens.data_ptr(), row_slots.data_ptr(), count,
             slot_length.data_ptr(), slot_prev.data_ptr(), int(slot_length.numel()), history_in.data_ptr(),
             history_out.data_ptr(), x.data_ptr(), residual.data_ptr(), workspace.data_ptr(), workspace.numel(),
             torch.cuda.current_stream().cuda_stream)
        return residual

    def apply_mlp(self, layer, residual, scale):
        """HadamardMlp.Apply over the rows of residual [count][dim], in place,
        on torch's current stream (ndl_mlp_apply)."""
        import torch

        call("ndl_mlp_apply", self._h, layer, residual.data_ptr(), int(residual.shape[0]), float(scale),
             torch.cuda.current_stream().cuda_stream)
        return residual

    def close(self):
        if getattr(self, "_h", None):
            lib().ndl_model_destroy(self._h)
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


__all__ = ["Model", "InvalidDataError", "NotSupportedError", "DENSE", "CQ", "PERMUTATION", "CQ_ROWS", "RAW"]
