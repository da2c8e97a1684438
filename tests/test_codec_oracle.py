"""The codec oracle (oracle/codec_oracle.py) and the codec's C ABI without a GPU.

The reference's codec tests need the real s2-pro codec file and are all
`#[ignore]` (codec.rs:3972-4060): they decode the codes below (2 frames of 10
codebooks) and assert shapes, finiteness and non-zero output.  Those checks
run here on the synthetic codec file.  The oracle's vectorised convolutions
are pinned against plain loops written the way the reference writes them
(codec.rs:3505-3574, 3576-3619, 2212-2293), and its WAV writer against
wav.rs:7-39 field by field.
"""
import ctypes
import re
import struct
from pathlib import Path

import numpy as np
import pytest

from oracle import codec_oracle as co

ROOT = Path(__file__).resolve().parent.parent

# codec.rs:3987-3990: 2 frames x 10 codebooks, codebook-major
FIXTURE_CODES = [3988, 29, 487, 925, 184, 865, 526, 924, 37, 12, 189, 460, 854, 549, 947, 935, 339, 39, 892, 855]


def test_fixture_codes_through_the_oracle(codec_oracle_weights):
    """codec.rs:3974-4061: rvq lookup, post module and upsample on the fixture codes."""
    w = codec_oracle_weights
    lat = co.rvq_lookup_codes(FIXTURE_CODES, 10, 2, w)
    assert lat.shape == (2, 1024) and np.isfinite(lat).all() and (np.abs(lat) > 0).any()
    post = co.post_module(lat, w)
    assert post.shape == (2, 1024) and np.isfinite(post).all() and (np.abs(post) > 0).any()
    hid = co.rvq_decode_latents(lat, w)
    assert hid.shape == (8, 1024) and np.isfinite(hid).all() and (np.abs(hid) > 0).any()


def test_oracle_rejects_bad_codes(codec_oracle_weights):
    w = codec_oracle_weights
    with pytest.raises(co.CodecOracleError, match="codebook count"):
        co.rvq_lookup_codes(FIXTURE_CODES[:18], 9, 2, w)
    with pytest.raises(co.CodecOracleError, match="non-negative"):
        co.rvq_lookup_codes([-1] + FIXTURE_CODES[1:], 10, 2, w)
    with pytest.raises(co.CodecOracleError, match="out of range"):
        co.rvq_lookup_codes([0, 0, 1024] + FIXTURE_CODES[3:], 10, 2, w)  # residual codebook 0, frame 0
    with pytest.raises(co.CodecOracleError, match="at least one frame"):
        co.post_module(np.zeros((0, 1024)), w)


def _conv_transpose_loop(x, weight, dims, bias, stride):
    kernel, out_ch, in_ch = dims
    F = x.shape[0]
    out = np.zeros((F * stride, out_ch))
    for f in range(F):
        for k in range(kernel):
            row = f * stride + k
            if row >= F * stride:
                continue
            for oc in range(out_ch):
                for ic in range(in_ch):
                    out[row, oc] += x[f, ic] * weight[k + kernel * (oc + out_ch * ic)]
    return out + bias


def _causal_conv_loop(x, weight, dims, bias, dilation):
    kernel, in_ch, out_ch = dims
    F = x.shape[0]
    size = (kernel - 1) * dilation + 1
    pad = size - 1
    xp = np.zeros((F + pad, in_ch))
    xp[pad:] = x
    xp = xp.astype(np.float32).astype(np.float16).astype(np.float64)
    out = np.zeros((F, out_ch))
    for t in range(F):
        for oc in range(out_ch):
            s = bias[oc]
            for tap in range(kernel):
                for ic in range(in_ch):
                    s += xp[t + tap * dilation, ic] * weight[tap + kernel * (ic + in_ch * oc)]
            out[t, oc] = s
    return out


@pytest.mark.parametrize("kernel,stride", [(2, 2), (4, 2), (16, 8), (3, 2)])
def test_conv_transpose_matches_reference_loop(kernel, stride):
    rng = np.random.default_rng(kernel * 10 + stride)
    F, cin, cout = 5, 6, 4
    x = rng.standard_normal((F, cin))
    w = rng.standard_normal(kernel * cout * cin)
    b = rng.standard_normal(cout)
    got = co.conv_transpose_1d(x, w, [kernel, cout, cin], b, stride)
    assert got.shape == (F * stride, cout)
    np.testing.assert_allclose(got, _conv_transpose_loop(x, w, [kernel, cout, cin], b, stride), rtol=1e-12,
                               atol=1e-12)


@pytest.mark.parametrize("kernel,dilation", [(7, 1), (7, 3), (7, 9), (1, 1), (3, 2)])
def test_causal_conv_matches_reference_loop(kernel, dilation):
    rng = np.random.default_rng(kernel * 10 + dilation)
    F, cin, cout = 20, 5, 3
    x = rng.standard_normal((F, cin))
    w = rng.standard_normal(kernel * cin * cout)
    b = rng.standard_normal(cout)
    got = co.causal_conv1d(x, w, [kernel, cin, cout], b, dilation)
    np.testing.assert_allclose(got, _causal_conv_loop(x, w, [kernel, cin, cout], b, dilation), rtol=1e-12,
                               atol=1e-12)


def test_depthwise_conv_and_layer_norm_match_reference_loops():
    rng = np.random.default_rng(3)
    F, C = 9, 4
    x = rng.standard_normal((F, C))
    w = rng.standard_normal(7 * C)
    b = rng.standard_normal(C)
    want = np.zeros((F, C))
    for t in range(F):
        for c in range(C):
            s = b[c]
            for k in range(7):
                src = t + k - 6
                if src >= 0:
                    s += x[src, c] * w[k + 7 * c]
            want[t, c] = s
    np.testing.assert_allclose(co.depthwise_causal_conv1d(x, w, b), want, rtol=1e-12, atol=1e-12)
    g, bb = rng.standard_normal(C), rng.standard_normal(C)
    ln = co.layer_norm(x, g, bb, 1e-6)
    for t in range(F):
        m = x[t].mean()
        v = ((x[t] - m) ** 2).mean()
        np.testing.assert_allclose(ln[t], (x[t] - m) / np.sqrt(v + 1e-6) * g + bb, rtol=1e-12)


def test_erf_approximation_is_close_to_erf():
    from math import erf
    xs = np.linspace(-4, 4, 101)
    got = co.erf_approx(xs)
    assert np.max(np.abs(got - np.array([erf(v) for v in xs]))) < 2e-7


def test_wav_writers_agree_with_the_reference_layout():
    from fish_s2pro_b200.codec import pcm_to_wav
    s = np.array([0.0, 0.5, -0.5, 1.5, -2.0, 0.99999, -0.00001], np.float32)
    a, b = co.pcm_to_wav(s), pcm_to_wav(s)
    assert a == b
    assert a[:4] == b"RIFF" and a[8:16] == b"WAVEfmt " and a[36:40] == b"data"
    riff, fmt_len, fmt, ch, rate, brate, align, bits = struct.unpack("<I4x4xIHHIIHH", a[4:36])
    assert (riff, fmt_len, fmt, ch, rate, brate, align, bits) == (44 + 14, 16, 1, 1, 44100, 88200, 2, 16)
    assert struct.unpack("<I", a[40:44])[0] == 14
    assert list(np.frombuffer(a[44:], "<i2")) == [0, 16383, -16383, 32767, -32767, 32766, 0]


def _header_symbols():
    text = (ROOT / "include" / "s2d_codec.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(s2d_codec_\w+)\s*\(", text)))


def test_library_exports_the_codec_entry_points():
    from fish_s2pro_b200 import build, codec, s2d
    build.build_runtime()
    lib = ctypes.CDLL(str(s2d.LIB_PATH))
    syms = _header_symbols()
    assert len(syms) == 15
    assert not [s for s in syms if not hasattr(lib, s)]
    assert sorted(codec.CODEC_SIGNATURES) == syms


def test_codec_open_reports_bad_files_without_a_gpu(tmp_path):
    from fish_s2pro_b200 import CodecDecoder, S2dError
    with pytest.raises(S2dError) as e:
        CodecDecoder.open(tmp_path / "missing.gguf")
    assert e.value.code == -2
    # a GGUF of another architecture
    p = tmp_path / "lm.gguf"
    key, val = b"general.architecture", b"fish-speech"
    p.write_bytes(b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + struct.pack("<Q", len(key)) + key +
                  struct.pack("<IQ", 8, len(val)) + val)
    with pytest.raises(S2dError, match="fish-speech-codec") as e:
        CodecDecoder.open(p)
    assert e.value.code == -1


def test_python_mirror_checks_lengths_before_the_library():
    from fish_s2pro_b200 import CodecDecoder, S2dError
    c = CodecDecoder(None)
    with pytest.raises(S2dError, match="codes length mismatch"):
        c.decode_waveform(FIXTURE_CODES, 10, 3)
    with pytest.raises(S2dError, match="post_module input length mismatch"):
        c.rvq_decode_latents(np.zeros(100, np.float32), 1)
    with pytest.raises(S2dError, match="decoder input length mismatch"):
        c.forward_codec_decoder(np.zeros(100, np.float32), 1)


# ---- reference-audio encoder ------------------------------------------------

def fixture_pcm(n=2048):
    """codec.rs:4194-4196 / 4264-4266: ((i % 97) - 48) / 4096."""
    return ((np.arange(n) % 97).astype(np.float32) - 48.0) / 4096.0


def _strided_conv_loop(x, weight, dims, bias, stride):
    """causal_conv_1d_frame_major (codec.rs:2212-2293) as the reference loops it."""
    kernel, in_ch, out_ch = dims
    F = x.shape[0]
    pad = kernel - stride
    n = np.ceil(np.float32(F - kernel + pad) / np.float32(stride) + np.float32(1.0))
    extra = max((max(int(n) - 1, 0)) * stride + (kernel - pad) - F, 0)
    xp = np.zeros((F + pad + extra, in_ch))
    xp[pad:pad + F] = x
    xp = xp.astype(np.float32).astype(np.float16).astype(np.float64)
    out = (xp.shape[0] - kernel) // stride + 1
    y = np.zeros((out, out_ch))
    for t in range(out):
        for oc in range(out_ch):
            s = bias[oc]
            for tap in range(kernel):
                src = t * stride + tap
                if src >= xp.shape[0]:
                    continue
                for ic in range(in_ch):
                    s += xp[src, ic] * weight[tap + kernel * (ic + in_ch * oc)]
            y[t, oc] = s
    return y


@pytest.mark.parametrize("kernel,stride,F", [(4, 2, 12), (16, 8, 32), (2, 2, 10), (4, 2, 7)])
def test_strided_conv_matches_reference_loop(kernel, stride, F):
    rng = np.random.default_rng(kernel + stride + F)
    cin, cout = 3, 4
    x = rng.standard_normal((F, cin))
    w = rng.standard_normal(kernel * cin * cout)
    b = rng.standard_normal(cout)
    got = co.causal_conv1d_strided(x, w, [kernel, cin, cout], b, stride)
    np.testing.assert_allclose(got, _strided_conv_loop(x, w, [kernel, cin, cout], b, stride), rtol=1e-12, atol=1e-12)


def test_fixture_pcm_through_the_oracle_encoder(codec_oracle_weights):
    """codec.rs:4189-4218 and 4258-4276: 2,048 samples -> 4 encoder frames -> 1
    quantizer frame of 10 in-range codes; codec.rs:4096-4122: 8 latent frames
    of ((i % 97) - 48) / 512 -> 2 frames through the quantizer encode stage."""
    w = codec_oracle_weights
    h, padded = co.forward_codec_encoder_frontend(fixture_pcm(), w)
    assert padded == 2048 and h.shape == (4, 1024) and np.isfinite(h).all() and (np.abs(h) > 0).any()
    codes, l2, enc_frames, q_frames, padded = co.encode_reference_audio(fixture_pcm(), w)
    assert (enc_frames, q_frames, padded) == (4, 1, 2048) and codes.shape == (10, 1)
    assert 0 <= codes[0, 0] < 4096 and all(0 <= c < 1024 for c in codes[1:, 0]) and np.isfinite(l2).all()
    lat = (((np.arange(8 * 1024) % 97) - 48.0) / 512.0).reshape(8, 1024)
    q = co.forward_codec_quantizer_encode_stage(lat, w)
    assert q.shape == (2, 1024) and np.isfinite(q).all() and (np.abs(q) > 0).any()
    assert co.pad_sample_count(0) == 2048 and co.pad_sample_count(2049) == 4096


def _wav(fmt, ch, rate, bits, data, extra_chunk=b""):
    fmt_chunk = struct.pack("<HHIIHH", fmt, ch, rate, rate * ch * bits // 8, ch * bits // 8, bits)
    body = b"WAVE" + extra_chunk + b"fmt " + struct.pack("<I", 16) + fmt_chunk + b"data" + \
        struct.pack("<I", len(data)) + data + (b"\0" if len(data) % 2 else b"")
    return b"RIFF" + struct.pack("<I", len(body)) + body


def test_wav_reader_follows_the_reference():
    """wav.rs:41-170: formats, odd-length chunks, channel averaging, errors."""
    from fish_s2pro_b200 import S2dError, read_wav_mono_f32
    from fish_s2pro_b200.codec import pcm_to_wav
    s = np.array([0.0, 0.5, -0.25, 0.999], np.float32)
    got = read_wav_mono_f32(pcm_to_wav(s))
    assert np.array_equal(got, (s * 32767).astype(np.int16).astype(np.float32) / 32768)
    assert np.array_equal(read_wav_mono_f32(_wav(1, 1, 44100, 8, bytes([0, 128, 255]))),
                          np.array([-1.0, 0.0, 127 / 128], np.float32))
    assert np.allclose(read_wav_mono_f32(_wav(1, 1, 44100, 24, bytes([0, 0, 0x80, 0xff, 0xff, 0x7f]))),
                       [-1.0, 8388607 / 8388608])
    assert np.array_equal(read_wav_mono_f32(_wav(3, 1, 44100, 32, np.array([0.25, -2.0], "<f4").tobytes())),
                          np.array([0.25, -2.0], np.float32))
    stereo = np.array([1000, 3000, -2000, 0], "<i2").tobytes()
    assert np.allclose(read_wav_mono_f32(_wav(1, 2, 44100, 16, stereo, extra_chunk=b"LIST\x03\0\0\0abc\0")),
                       [2000 / 32768, -1000 / 32768])
    with pytest.raises(S2dError, match="expected 44100 Hz"):
        read_wav_mono_f32(_wav(1, 1, 16000, 16, b"\0\0"))
    with pytest.raises(S2dError, match="unsupported WAV format"):
        read_wav_mono_f32(_wav(1, 1, 44100, 12, b"\0\0"))
    with pytest.raises(S2dError, match="no samples"):
        read_wav_mono_f32(_wav(1, 1, 44100, 16, b""))
    with pytest.raises(S2dError, match="not a RIFF"):
        read_wav_mono_f32(b"RIFX0000WAVE")
