"""Codec decode on the GPU: RVQ codes -> 44.1 kHz PCM (include/s2d_codec.h).

Mirrors the reference's codec API (crates/fish_s2_infer/src/codec.rs):
`rvq_lookup_codes` (2536), `rvq_decode_latents` (1282),
`forward_codec_decoder` (1941), `decode_waveform` (1690) and
`decode_waveform_to_wav` (1716), with the reference's result records, over
one handle that holds the codec's decode weights in HBM.  Errors raise
S2dError with the reference's messages where it has one.
"""
from __future__ import annotations

import ctypes
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .s2d import S2dError, lib

_P = ctypes.POINTER
_c = ctypes
CODEC_SAMPLE_RATE = 44100  # codec.rs:55
CODEC_HIDDEN_SIZE = 1024
SAMPLES_PER_FRAME = 2048   # 2 x 2 upsample, 8 x 8 x 4 x 2 decoder

CODEC_SIGNATURES = {
    "s2d_codec_open": (_c.c_int32, [_c.c_char_p, _c.c_int32, _P(_c.c_void_p)]),
    "s2d_codec_close": (None, [_c.c_void_p]),
    "s2d_codec_last_error": (_c.c_char_p, [_c.c_void_p]),
    "s2d_codec_decode_waveform": (_c.c_int32, [_c.c_void_p, _P(_c.c_int32), _c.c_uint32, _c.c_uint32,
                                               _P(_c.c_float), _c.c_size_t, _P(_c.c_size_t), _P(_c.c_uint32)]),
    "s2d_codec_decode_waveform_device": (_c.c_int32, [_c.c_void_p, _c.c_void_p, _c.c_uint32, _c.c_uint32,
                                                      _c.c_void_p, _c.c_void_p]),
    "s2d_codec_sync": (_c.c_int32, [_c.c_void_p]),
    "s2d_codec_rvq_lookup": (_c.c_int32, [_c.c_void_p, _P(_c.c_int32), _c.c_uint32, _c.c_uint32,
                                          _P(_c.c_float)]),
    "s2d_codec_decode_latents": (_c.c_int32, [_c.c_void_p, _P(_c.c_float), _c.c_uint32, _P(_c.c_float)]),
    "s2d_codec_decoder": (_c.c_int32, [_c.c_void_p, _P(_c.c_float), _c.c_uint32, _c.c_uint32, _P(_c.c_float)]),
    "s2d_codec_memory": (_c.c_int32, [_c.c_void_p, _P(_c.c_size_t), _P(_c.c_size_t)]),
}

_bound = False


def codec_lib() -> ctypes.CDLL:
    """libs2d.so with the codec entry points typed."""
    global _bound
    l = lib()
    if not _bound:
        for name, (res, args) in CODEC_SIGNATURES.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _bound = True
    return l


@dataclass
class CodecRvqLookupResult:  # codec.rs:2514
    num_codebooks: int
    n_frames: int
    latent_dim: int
    latents: np.ndarray


@dataclass
class CodecDecodeLatentsResult:  # codec.rs:1275
    input_frames: int
    output_frames: int
    hidden_dim: int
    hidden: np.ndarray


@dataclass
class CodecWaveformResult:  # codec.rs:1681
    sample_rate: int
    input_frames: int
    latent_frames: int
    num_samples: int
    samples: np.ndarray


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32).reshape(-1))


def _codes(codes) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(codes, dtype=np.int32).reshape(-1))


class CodecDecoder:
    """The codec's decode weights on one GPU (s2d_codec_open)."""

    def __init__(self, handle):
        self.handle = handle

    @classmethod
    def open(cls, gguf_path: str | Path, device: int = 0) -> "CodecDecoder":
        l = codec_lib()
        h = ctypes.c_void_p()
        rc = l.s2d_codec_open(str(gguf_path).encode(), device, ctypes.byref(h))
        if rc != 0:
            msg = l.s2d_codec_last_error(h).decode() if h else "s2d_codec_open failed"
            l.s2d_codec_close(h)
            raise S2dError(rc, msg)
        return cls(h)

    def close(self) -> None:
        if self.handle:
            codec_lib().s2d_codec_close(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, rc: int) -> None:
        if rc != 0:
            raise S2dError(rc, codec_lib().s2d_codec_last_error(self.handle).decode())

    def rvq_lookup_codes(self, codes, num_codebooks: int, n_frames: int) -> CodecRvqLookupResult:
        c = _codes(codes)
        if c.size != num_codebooks * n_frames:
            raise S2dError(-1, f"codec codes length mismatch: expected {num_codebooks * n_frames}, got {c.size}")
        out = np.empty(n_frames * CODEC_HIDDEN_SIZE, np.float32)
        self._check(codec_lib().s2d_codec_rvq_lookup(self.handle, c.ctypes.data_as(_P(_c.c_int32)), num_codebooks,
                                                     n_frames, out.ctypes.data_as(_P(_c.c_float))))
        return CodecRvqLookupResult(num_codebooks, n_frames, CODEC_HIDDEN_SIZE, out)

    def rvq_decode_latents(self, latents, n_frames: int) -> CodecDecodeLatentsResult:
        x = _f32(latents)
        if x.size != n_frames * CODEC_HIDDEN_SIZE:
            raise S2dError(-1, f"post_module input length mismatch: expected {n_frames * CODEC_HIDDEN_SIZE}, "
                               f"got {x.size}")
        out = np.empty(4 * n_frames * CODEC_HIDDEN_SIZE, np.float32)
        self._check(codec_lib().s2d_codec_decode_latents(self.handle, x.ctypes.data_as(_P(_c.c_float)), n_frames,
                                                         out.ctypes.data_as(_P(_c.c_float))))
        return CodecDecodeLatentsResult(n_frames, 4 * n_frames, CODEC_HIDDEN_SIZE, out)

    def forward_codec_decoder(self, hidden, n_frames: int, hidden_dim: int = CODEC_HIDDEN_SIZE) -> np.ndarray:
        x = _f32(hidden)
        if x.size != n_frames * hidden_dim:
            raise S2dError(-1, f"decoder input length mismatch: expected {n_frames * hidden_dim}, got {x.size}")
        out = np.empty(n_frames * SAMPLES_PER_FRAME // 4, np.float32)
        self._check(codec_lib().s2d_codec_decoder(self.handle, x.ctypes.data_as(_P(_c.c_float)), n_frames,
                                                  hidden_dim, out.ctypes.data_as(_P(_c.c_float))))
        return out

    def decode_waveform(self, codes, num_codebooks: int, n_frames: int) -> CodecWaveformResult:
        c = _codes(codes)
        if c.size != num_codebooks * n_frames:
            raise S2dError(-1, f"codec codes length mismatch: expected {num_codebooks * n_frames}, got {c.size}")
        out = np.empty(max(1, n_frames) * SAMPLES_PER_FRAME, np.float32)
        n = ctypes.c_size_t()
        lat = ctypes.c_uint32()
        self._check(codec_lib().s2d_codec_decode_waveform(
            self.handle, c.ctypes.data_as(_P(_c.c_int32)), num_codebooks, n_frames,
            out.ctypes.data_as(_P(_c.c_float)), out.size, ctypes.byref(n), ctypes.byref(lat)))
        return CodecWaveformResult(CODEC_SAMPLE_RATE, n_frames, lat.value, n.value, out[:n.value])

    def decode_waveform_to_wav(self, codes, num_codebooks: int, n_frames: int) -> bytes:
        w = self.decode_waveform(codes, num_codebooks, n_frames)
        return pcm_to_wav(w.samples, w.sample_rate)

    def memory(self) -> tuple[int, int]:
        wb, ws = ctypes.c_size_t(), ctypes.c_size_t()
        self._check(codec_lib().s2d_codec_memory(self.handle, ctypes.byref(wb), ctypes.byref(ws)))
        return wb.value, ws.value


def pcm_to_wav(samples, sample_rate: int = CODEC_SAMPLE_RATE) -> bytes:
    """wav.rs:7 pcm_to_wav: 44-byte RIFF header, 16-bit mono PCM, each sample
    clamped to [-1, 1], scaled by 32767 and truncated toward zero."""
    s = np.clip(np.asarray(samples, np.float32), np.float32(-1.0), np.float32(1.0))
    pcm = (s * np.float32(32767.0)).astype(np.int16)
    n = pcm.size
    hdr = (b"RIFF" + struct.pack("<I", 44 + 2 * n) + b"WAVEfmt " +
           struct.pack("<IHHIIHH", 16, 1, 1, sample_rate, sample_rate * 2, 2, 16) + b"data" + struct.pack("<I", 2 * n))
    return hdr + pcm.astype("<i2").tobytes()
