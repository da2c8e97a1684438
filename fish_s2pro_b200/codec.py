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
    "s2d_codec_has_encoder": (_c.c_int32, [_c.c_void_p]),
    "s2d_codec_encode_reference_audio": (_c.c_int32, [_c.c_void_p, _P(_c.c_float), _c.c_size_t, _P(_c.c_int32),
                                                      _c.c_size_t, _P(_c.c_uint32), _P(_c.c_uint32),
                                                      _P(_c.c_uint32), _P(_c.c_float)]),
    "s2d_codec_encoder_frontend": (_c.c_int32, [_c.c_void_p, _P(_c.c_float), _c.c_size_t, _P(_c.c_float),
                                                _c.c_size_t, _P(_c.c_uint32), _P(_c.c_uint32)]),
    "s2d_codec_quantizer_encode": (_c.c_int32, [_c.c_void_p, _P(_c.c_float), _c.c_uint32, _P(_c.c_float)]),
    "s2d_codec_vq_encode": (_c.c_int32, [_c.c_void_p, _P(_c.c_float), _c.c_uint32, _P(_c.c_int32),
                                         _P(_c.c_float)]),
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


@dataclass
class CodecReferenceAudioResult:  # codec.rs:955
    input_samples: int
    padded_samples: int
    encoder_frames: int
    quantizer_frames: int
    num_codebooks: int
    codes: np.ndarray
    final_residual_l2: np.ndarray


@dataclass
class CodecEncoderFrontendResult:  # codec.rs:966
    input_samples: int
    padded_samples: int
    output_frames: int
    hidden_dim: int
    hidden: np.ndarray


@dataclass
class CodecEncodeStageResult:  # codec.rs:927
    input_frames: int
    output_frames: int
    hidden_dim: int
    hidden: np.ndarray


@dataclass
class CodecVqEncodeResult:  # codec.rs:2522
    num_codebooks: int
    n_frames: int
    latent_dim: int
    codes: np.ndarray
    final_residual_l2: np.ndarray


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32).reshape(-1))


def _codes(codes) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(codes, dtype=np.int32).reshape(-1))


class Codec:
    """The codec on one GPU (s2d_codec_open): decode (codes -> PCM) and, when
    the file holds it, the reference-audio encoder (PCM -> prompt codes)."""

    def __init__(self, handle):
        self.handle = handle

    @classmethod
    def open(cls, gguf_path: str | Path, device: int = 0) -> "Codec":
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

    # ---- reference-audio encoder (codec.rs:1056-1086) ----

    @property
    def has_encoder(self) -> bool:
        return bool(codec_lib().s2d_codec_has_encoder(self.handle))

    def encode_reference_audio(self, audio) -> CodecReferenceAudioResult:
        a = _f32(audio)
        frames = max(1, (a.size + SAMPLES_PER_FRAME - 1) // SAMPLES_PER_FRAME)
        codes = np.empty(10 * frames, np.int32)
        l2 = np.empty(frames, np.float32)
        q, e, p = ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint32()
        self._check(codec_lib().s2d_codec_encode_reference_audio(
            self.handle, a.ctypes.data_as(_P(_c.c_float)), a.size, codes.ctypes.data_as(_P(_c.c_int32)), codes.size,
            ctypes.byref(q), ctypes.byref(e), ctypes.byref(p), l2.ctypes.data_as(_P(_c.c_float))))
        return CodecReferenceAudioResult(a.size, p.value, e.value, q.value, 10, codes, l2)

    def encode_reference_wav_file(self, path) -> CodecReferenceAudioResult:
        return self.encode_reference_audio(read_wav_mono_f32(path, CODEC_SAMPLE_RATE))

    def forward_codec_encoder_frontend(self, audio) -> CodecEncoderFrontendResult:
        a = _f32(audio)
        padded = max(1, (a.size + SAMPLES_PER_FRAME - 1) // SAMPLES_PER_FRAME) * SAMPLES_PER_FRAME
        out = np.empty(padded // 512 * CODEC_HIDDEN_SIZE, np.float32)
        f, p = ctypes.c_uint32(), ctypes.c_uint32()
        self._check(codec_lib().s2d_codec_encoder_frontend(
            self.handle, a.ctypes.data_as(_P(_c.c_float)), a.size, out.ctypes.data_as(_P(_c.c_float)), out.size,
            ctypes.byref(f), ctypes.byref(p)))
        return CodecEncoderFrontendResult(a.size, p.value, f.value, CODEC_HIDDEN_SIZE, out)

    def forward_codec_quantizer_encode_stage(self, hidden, n_frames: int) -> CodecEncodeStageResult:
        x = _f32(hidden)
        if x.size != n_frames * CODEC_HIDDEN_SIZE:
            raise S2dError(-1, f"codec quantizer encode input length mismatch: expected "
                               f"{n_frames * CODEC_HIDDEN_SIZE}, got {x.size}")
        out = np.empty(n_frames // 4 * CODEC_HIDDEN_SIZE, np.float32)
        self._check(codec_lib().s2d_codec_quantizer_encode(self.handle, x.ctypes.data_as(_P(_c.c_float)), n_frames,
                                                           out.ctypes.data_as(_P(_c.c_float))))
        return CodecEncodeStageResult(n_frames, n_frames // 4, CODEC_HIDDEN_SIZE, out)

    def rvq_encode_latents_nearest(self, latents, n_frames: int) -> CodecVqEncodeResult:
        x = _f32(latents)
        if x.size != n_frames * CODEC_HIDDEN_SIZE:
            raise S2dError(-1, f"codec VQ encode input length mismatch: expected {n_frames * CODEC_HIDDEN_SIZE}, "
                               f"got {x.size}")
        codes = np.empty(10 * n_frames, np.int32)
        l2 = np.empty(n_frames, np.float32)
        self._check(codec_lib().s2d_codec_vq_encode(self.handle, x.ctypes.data_as(_P(_c.c_float)), n_frames,
                                                    codes.ctypes.data_as(_P(_c.c_int32)),
                                                    l2.ctypes.data_as(_P(_c.c_float))))
        return CodecVqEncodeResult(10, n_frames, CODEC_HIDDEN_SIZE, codes, l2)

    def memory(self) -> tuple[int, int]:
        wb, ws = ctypes.c_size_t(), ctypes.c_size_t()
        self._check(codec_lib().s2d_codec_memory(self.handle, ctypes.byref(wb), ctypes.byref(ws)))
        return wb.value, ws.value


CodecDecoder = Codec  # the decode-side name


def read_wav_mono_f32(path_or_bytes, expected_sample_rate: int = CODEC_SAMPLE_RATE) -> np.ndarray:
    """wav.rs:41-170 read_wav_mono_f32: RIFF/WAVE chunks (fmt, data; odd
    chunks padded), PCM 8 / 16 / 24 / 32-bit or IEEE float 32, channels
    averaged to mono; the sample rate must match."""
    b = Path(path_or_bytes).read_bytes() if not isinstance(path_or_bytes, (bytes, bytearray)) else bytes(path_or_bytes)
    if len(b) < 12 or b[0:4] != b"RIFF" or b[8:12] != b"WAVE":
        raise S2dError(-1, "not a RIFF/WAVE file")
    off, fmt, data = 12, None, None
    while off + 8 <= len(b):
        cid, n = b[off:off + 4], struct.unpack_from("<I", b, off + 4)[0]
        off += 8
        end = off + n
        if end > len(b):
            raise S2dError(-1, "WAV chunk extends past file end")
        if cid == b"fmt ":
            if n < 16:
                raise S2dError(-1, "WAV fmt chunk too short")
            af, ch, rate = struct.unpack_from("<HHI", b, off)
            bits = struct.unpack_from("<H", b, off + 14)[0]
            fmt = (af, ch, rate, bits)
        elif cid == b"data":
            data = b[off:end]
        off = end + (n % 2)
    if fmt is None:
        raise S2dError(-1, "missing WAV fmt chunk")
    if data is None:
        raise S2dError(-1, "missing WAV data chunk")
    af, ch, rate, bits = fmt
    if ch == 0:
        raise S2dError(-1, "WAV has zero channels")
    if rate != expected_sample_rate:
        raise S2dError(-1, f"expected {expected_sample_rate} Hz WAV, got {rate} Hz")
    width = {(1, 8): 1, (1, 16): 2, (1, 24): 3, (1, 32): 4, (3, 32): 4}.get((af, bits))
    if width is None:
        raise S2dError(-1, f"unsupported WAV format: audio_format={af}, bits_per_sample={bits}")
    if len(data) % width:
        raise S2dError(-1, f"WAV data length is not divisible by {width}")
    if (af, bits) == (1, 8):
        x = (np.frombuffer(data, np.uint8).astype(np.float32) - np.float32(128.0)) / np.float32(128.0)
    elif (af, bits) == (1, 16):
        x = np.frombuffer(data, "<i2").astype(np.float32) / np.float32(32768.0)
    elif (af, bits) == (1, 24):
        u = np.frombuffer(data, np.uint8).reshape(-1, 3).astype(np.int32)
        v = u[:, 0] | (u[:, 1] << 8) | (u[:, 2] << 16)
        v = np.where(v & 0x800000, v - (1 << 24), v)
        x = v.astype(np.float32) / np.float32(8388608.0)
    elif (af, bits) == (1, 32):
        x = np.frombuffer(data, "<i4").astype(np.float32) / np.float32(2147483648.0)
    else:
        x = np.frombuffer(data, "<f4").astype(np.float32)
    if x.size == 0:
        raise S2dError(-1, "WAV contains no samples")
    if ch == 1:
        return x
    if x.size % ch:
        raise S2dError(-1, "WAV sample count is not divisible by channel count")
    frames = x.reshape(-1, ch)
    out = frames[:, 0].copy()
    for j in range(1, ch):
        out = (out + frames[:, j]).astype(np.float32)
    return (out / np.float32(ch)).astype(np.float32)


def pcm_to_wav(samples, sample_rate: int = CODEC_SAMPLE_RATE) -> bytes:
    """wav.rs:7 pcm_to_wav: 44-byte RIFF header, 16-bit mono PCM, each sample
    clamped to [-1, 1], scaled by 32767 and truncated toward zero."""
    s = np.clip(np.asarray(samples, np.float32), np.float32(-1.0), np.float32(1.0))
    pcm = (s * np.float32(32767.0)).astype(np.int16)
    n = pcm.size
    hdr = (b"RIFF" + struct.pack("<I", 44 + 2 * n) + b"WAVEfmt " +
           struct.pack("<IHHIIHH", 16, 1, 1, sample_rate, sample_rate * 2, 2, 16) + b"data" + struct.pack("<I", 2 * n))
    return hdr + pcm.astype("<i2").tobytes()
