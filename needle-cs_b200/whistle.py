"""Whistle: the speech encoder of a Needle-3 archive with an audio section,
on the GPU (ndl_whistle_*).  Mirrors the reference's Whistle encoder surface
(src/Needle/Whistle.cs: Encode, Embed, Frames, and the cross memory that
BuildCrossMemory attaches to the decoder)."""
import ctypes

import numpy as np

from ._native import call, lib

MEL, STEM, ENCODER, KEYS, KEY_SCALES, VALUES, VALUE_SCALES = range(7)


class Whistle:
    """`model` a loaded needle_cs_b200.model.Model on a device; `max_seconds`
    bounds the audio per call (the reference keeps at most 30 s)."""

    MaxSeconds = 30

    def __init__(self, model, max_seconds=MaxSeconds):
        self.model = model
        info = model.info
        self.dim, self.heads, self.qk, self.vd = info["dim"], info["heads"], info["qk_dim"], info["v_dim"]
        self.layers = info["layers"]
        manifest = np.asarray(model.host("audio", 0), np.float32)
        self.mels, self.sample_rate, self.hop = int(manifest[8]), int(manifest[9]), int(manifest[12])
        h = ctypes.c_void_p()
        call("ndl_whistle_create", model._h, int(max_seconds * self.sample_rate), ctypes.byref(h))
        self._h = h
        self.frames = 0

    def close(self):
        if self._h:
            call("ndl_whistle_destroy", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def encode(self, pcm):
        """Whistle.Encode: the encoder over `pcm` (float32 samples) and the cross
        memory of every decoder layer; returns the frame count."""
        pcm = np.ascontiguousarray(pcm, np.float32)
        frames = ctypes.c_int()
        call("ndl_whistle_encode", self._h, pcm.ctypes.data, pcm.size, ctypes.byref(frames))
        self.frames = frames.value
        return self.frames

    def _read(self, what, dtype, shape, layer=0):
        out = np.empty(shape, dtype)
        call("ndl_whistle_read", self._h, what, layer, out.ctypes.data, out.nbytes, None)
        return out

    def mel(self):
        """The normalized log-mel features [mel frames][mels]."""
        mel_frames = ctypes.c_int()
        call("ndl_whistle_frames", self._h, None, ctypes.byref(mel_frames))
        return self._read(MEL, np.float32, (mel_frames.value, self.mels))

    def stem(self):
        return self._read(STEM, np.float32, (self.frames, self.dim))

    def encoder_output(self):
        return self._read(ENCODER, np.float32, (self.frames, self.dim))

    def embed(self, pcm):
        """Whistle.Embed: the encoder output rows [frames][dim]."""
        self.encode(pcm)
        return self.encoder_output()

    def memory(self, layer):
        """(keys int8 [frames][heads * qk], key scales [frames][heads], values int8
        [frames][heads * v], value scales [frames][heads]) of decoder `layer`."""
        F, H = self.frames, self.heads
        return (self._read(KEYS, np.int8, (F, H * self.qk), layer), self._read(KEY_SCALES, np.float32, (F, H), layer),
                self._read(VALUES, np.int8, (F, H * self.vd), layer),
                self._read(VALUE_SCALES, np.float32, (F, H), layer))

    def stream(self):
        """The cudaStream_t the encoder's kernels run on."""
        return lib().ndl_whistle_stream(self._h)
