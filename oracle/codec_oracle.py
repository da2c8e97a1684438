"""CPU restatement of the reference's codec decode (codes -> 44.1 kHz PCM).

TEST INFRASTRUCTURE ONLY: the parity checker for the sm_100a codec path and
the codec's timed CPU baseline.  Only tests/ and bench.py's CPU legs use it;
nothing in fish_s2pro_b200 imports it.

Every function restates the reference function named in its docstring
(crates/fish_s2_infer/src/codec.rs unless stated otherwise) with numpy in
float64, vectorised over frames; where the reference rounds a value to f16
(the causal convolutions' padded input, codec.rs:2257-2259) this does the
same rounding from the float32 value.  Parity of the oracle itself is
unpinned: the reference's codec tests need the real s2-pro codec file
(codec.rs:3972-4060, all `#[ignore]`), so there are no golden vectors; the
structural facts those tests assert (2 frames -> 8 latent frames, finite,
non-zero) are checked in tests/test_codec_oracle.py.
"""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np

# codec.rs:16-55
HIDDEN = 1024
PROJ = 8
SEMANTIC_CODEBOOK = 4096
RESIDUAL_CODEBOOK = 1024
RESIDUAL_QUANTIZERS = 9
LAYERS = 8
FFN = 3072
HEAD_DIM = 64
HEADS = 16
ROPE_BASE = 10000.0
NORM_EPS = 1e-5
WINDOW = 128
UPSAMPLE_STAGES = 2
UPSAMPLE_FACTOR = 2
CONVNEXT_KERNEL = 7
CONVNEXT_EXPANDED = 4096
CONVNEXT_EPS = 1e-6
LATENT_DIM = 1024
DECODER_ENTRY_CHANNELS = 1536
DECODER_RATES = (8, 8, 4, 2)
DECODER_CHANNELS = (768, 384, 192, 96)  # block_output_channels, codec.rs:2003-2012
SAMPLE_RATE = 44100


class CodecOracleError(RuntimeError):
    pass


# ---- GGUF (F16 / F32 tensors only; crates/fish_s2_core/src/gguf.rs) ---------

_GGUF_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q",
                12: "<d"}


def read_gguf(path):
    """(metadata dict, {name: (ggml dims, flat f16 / f32 array)}) of a GGUF
    v3 file; tensors of other types are skipped."""
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    data = bytes(mm[:min(mm.size, 4 << 20)])  # the header (tensor directory) lies in the first MiB
    off = 0

    def take(fmt):
        nonlocal off
        v = struct.unpack_from(fmt, data, off)[0]
        off += struct.calcsize(fmt)
        return v

    def string():
        nonlocal off
        n = take("<Q")
        s = data[off:off + n].decode()
        off += n
        return s

    def value(t):
        if t in _GGUF_SCALAR:
            return take(_GGUF_SCALAR[t])
        if t == 8:
            return string()
        if t == 9:
            et, n = take("<I"), take("<Q")
            return [value(et) for _ in range(n)]
        raise CodecOracleError(f"unknown GGUF metadata type {t}")

    if data[:4] != b"GGUF":
        raise CodecOracleError("not a GGUF file")
    off = 4
    version, n_tensors, n_meta = take("<I"), take("<Q"), take("<Q")
    if version != 3:
        raise CodecOracleError(f"GGUF version {version}")
    meta = {}
    for _ in range(n_meta):
        k = string()
        meta[k] = value(take("<I"))
    infos = []
    for _ in range(n_tensors):
        name = string()
        nd = take("<I")
        dims = [take("<Q") for _ in range(nd)]
        infos.append((name, dims, take("<I"), take("<Q")))
    align = int(meta.get("general.alignment", 32))
    start = (off + align - 1) // align * align
    tensors = {}
    for name, dims, t, rel in infos:
        n = int(np.prod(dims))
        o = start + rel
        if t == 1:
            a = mm[o:o + 2 * n].view(np.float16)
        elif t == 0:
            a = mm[o:o + 4 * n].view(np.float32)
        else:
            continue
        tensors[name] = (dims, a)
    return meta, tensors


def f16_to_f32(a):
    """IEEE half -> float by bit manipulation (numpy's own f16 cast is slow
    for hundreds of millions of values); exact for every f16 value."""
    h = np.asarray(a).view(np.uint16).astype(np.uint32)
    sign = (h & 0x8000) << 16
    e = (h >> 10) & 0x1F
    m = h & 0x3FF
    normal = (sign | ((e + 112) << 23) | (m << 13)).view(np.float32)
    special = (sign | 0x7F800000 | (m << 13)).view(np.float32)
    sub = (m.astype(np.float32) * np.float32(2.0 ** -24)) * np.where(sign != 0, np.float32(-1), np.float32(1))
    return np.where(e == 0, sub, np.where(e == 31, special, normal))


class CodecWeights:
    """The decode tensors of a codec GGUF, by the reference's names
    (codec.rs:277-297 quantizers, 315-333 transformer layers, 429-447
    upsample stages, 1308-1320 residual units, 1403-1440 decoder)."""

    def __init__(self, path, dtype=np.float64):
        """dtype: the arithmetic of every stage (float64 for the parity
        reference; float32 restates the reference's own precision)."""
        self.dtype = dtype
        meta, self.t = read_gguf(path)
        if meta.get("general.architecture") != "fish-speech-codec":
            raise CodecOracleError("expected fish-speech-codec codec GGUF")
        self._f64 = {}

    def get(self, name, dims=None):
        """The tensor as a flat array of self.dtype (converted on first use)."""
        if name not in self.t:
            raise CodecOracleError(f"tensor not found: {name}")
        d, a = self.t[name]
        if dims is not None and list(d) != list(dims):
            raise CodecOracleError(f"{name}: expected {dims}, got {d}")
        if name not in self._f64:
            self._f64[name] = (f16_to_f32(a) if a.dtype == np.float16 else np.asarray(a)).astype(self.dtype)
        return self._f64[name]

    def quantizer(self, cb):
        p = "quantizer.semantic_quantizer.quantizers.0" if cb == 0 else f"quantizer.quantizer.quantizers.{cb - 1}"
        n = SEMANTIC_CODEBOOK if cb == 0 else RESIDUAL_CODEBOOK
        return (self.get(f"{p}.codebook.weight", [PROJ, n]).reshape(n, PROJ),
                self.get(f"{p}.out_proj.weight", [1, PROJ, HIDDEN]).reshape(HIDDEN, PROJ),
                self.get(f"{p}.out_proj.bias", [HIDDEN]))


# ---- RVQ lookup (codec.rs:2536-2596, project_code 2428-2445) ----------------

def rvq_lookup_codes(codes, num_codebooks, n_frames, w: CodecWeights):
    """latents [n_frames][1024]: per frame, the sum over codebooks of
    out_proj . codebook[code] + out_proj_bias (codec.rs:2536)."""
    codes = np.asarray(codes, np.int64)
    if num_codebooks != 1 + RESIDUAL_QUANTIZERS:
        raise CodecOracleError("codec codebook count mismatch")
    if codes.size != num_codebooks * n_frames:
        raise CodecOracleError("codec codes length mismatch")
    codes = codes.reshape(num_codebooks, n_frames)
    if (codes < 0).any():
        raise CodecOracleError("codec code must be non-negative")
    lat = np.zeros((n_frames, HIDDEN))
    for cb in range(num_codebooks):
        book, wo, bo = w.quantizer(cb)
        if (codes[cb] >= book.shape[0]).any():
            raise CodecOracleError("codec code out of range")
        lat += book[codes[cb]] @ wo.T + bo
    return lat


# ---- post module transformer (codec.rs:986-1018, 3229-3336) -----------------

def rms_norm(x, w, eps):
    """tensor.rs:155 rms_norm over the last axis."""
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * w


def rope_normal(x, position):
    """attention.rs:172 apply_rope_normal: adjacent pairs of each 64-wide head,
    theta = position / base^(pair / head_dim); x [T][n_heads * 64], position [T]."""
    T = x.shape[0]
    xh = x.reshape(T, -1, HEAD_DIM // 2, 2)
    pair = np.arange(0, HEAD_DIM, 2, dtype=np.float32) / np.float32(HEAD_DIM)
    inv = (np.float32(ROPE_BASE) ** pair).astype(np.float32)
    theta = (np.asarray(position, np.float32)[:, None] / inv[None, :]).astype(np.float64)
    c, s = np.cos(theta)[:, None, :], np.sin(theta)[:, None, :]
    x0, x1 = xh[..., 0], xh[..., 1]
    return np.stack([x0 * c - x1 * s, x0 * s + x1 * c], axis=-1).reshape(x.shape)


def windowed_attention(q, k, v, window=WINDOW):
    """The attention of codec.rs:3270-3297: query t over keys
    max(0, t + 1 - window) .. t (gqa_decode_attention, attention.rs:208, with
    16 heads of 64 and one head per KV group, scale 1 / 8)."""
    T = q.shape[0]
    qh, kh, vh = (a.reshape(T, HEADS, HEAD_DIM) for a in (q, k, v))
    out = np.zeros_like(qh)
    scale = 1.0 / np.sqrt(HEAD_DIM)
    for t in range(T):
        lo = max(0, t + 1 - window)
        s = np.einsum("hd,phd->hp", qh[t], kh[lo:t + 1]) * scale
        p = np.exp(s - s.max(axis=1, keepdims=True))
        p /= p.sum(axis=1, keepdims=True)
        out[t] = np.einsum("hp,phd->hd", p, vh[lo:t + 1])
    return out.reshape(T, HIDDEN)


def silu(x):
    return x / (1.0 + np.exp(-x))


def transformer_layer(x, w: CodecWeights, layer, module="quantizer.post_module", window=WINDOW):
    """codec.rs:3229 forward_codec_transformer_layer_with_window (window 128
    for the post and pre modules, 512 in the encoder)."""
    p = f"{module}.layers.{layer}"
    T = x.shape[0]
    h = rms_norm(x, w.get(f"{p}.attention_norm.weight", [HIDDEN]), NORM_EPS)
    qkv = h @ w.get(f"{p}.attention.wqkv.weight", [HIDDEN, 3 * HIDDEN]).reshape(3 * HIDDEN, HIDDEN).T
    q, k, v = qkv[:, :HIDDEN], qkv[:, HIDDEN:2 * HIDDEN], qkv[:, 2 * HIDDEN:]
    pos = np.arange(T)
    att = windowed_attention(rope_normal(q, pos), rope_normal(k, pos), v, window)
    o = att @ w.get(f"{p}.attention.wo.weight", [HIDDEN, HIDDEN]).reshape(HIDDEN, HIDDEN).T
    x = x + o * w.get(f"{p}.attention_layer_scale.gamma", [HIDDEN])
    h = rms_norm(x, w.get(f"{p}.ffn_norm.weight", [HIDDEN]), NORM_EPS)
    g = h @ w.get(f"{p}.feed_forward.w1.weight", [HIDDEN, FFN]).reshape(FFN, HIDDEN).T
    u = h @ w.get(f"{p}.feed_forward.w3.weight", [HIDDEN, FFN]).reshape(FFN, HIDDEN).T
    f = (silu(g) * u) @ w.get(f"{p}.feed_forward.w2.weight", [FFN, HIDDEN]).reshape(HIDDEN, FFN).T
    return x + f * w.get(f"{p}.ffn_layer_scale.gamma", [HIDDEN])


def post_module(lat, w: CodecWeights):
    """codec.rs:986 forward_codec_post_module: 8 layers, then the final RMSNorm."""
    if lat.shape[0] == 0:
        raise CodecOracleError("codec transformer requires at least one frame")
    x = lat
    for layer in range(LAYERS):
        x = transformer_layer(x, w, layer)
    return rms_norm(x, w.get("quantizer.post_module.norm.weight", [HIDDEN]), NORM_EPS)


# ---- upsample: transposed conv + ConvNeXt (codec.rs:2302, 3338, 3438) -------

def conv_transpose_1d(x, weight, dims, bias, stride):
    """codec.rs:3505 causal_conv_transpose_1d: weight ggml [kernel, out, in];
    out[f * stride + k] += W[k] . x[f]; rows past frames * stride dropped."""
    kernel, out_ch, in_ch = dims
    W = weight.reshape(in_ch, out_ch, kernel)
    F = x.shape[0]
    y = np.zeros((F * stride + kernel, out_ch), x.dtype)
    for k in range(kernel):
        y[k:k + F * stride:stride] += x @ W[:, :, k]
    return y[:F * stride] + bias


def depthwise_causal_conv1d(x, weight, bias, kernel=CONVNEXT_KERNEL):
    """codec.rs:3576: out[t][c] = b[c] + sum_k x[t + k - (kernel - 1)][c] W[c][k]."""
    F, C = x.shape
    W = weight.reshape(C, kernel)
    xp = np.concatenate([np.zeros((kernel - 1, C), x.dtype), x])
    y = np.tile(bias, (F, 1))
    for k in range(kernel):
        y += xp[k:k + F] * W[:, k]
    return y


def layer_norm(x, w, b, eps):
    """codec.rs:3621 layer_norm_affine_frame_major."""
    mu = x.mean(axis=-1, keepdims=True)
    var = ((x - mu) ** 2).mean(axis=-1, keepdims=True)
    return (x - mu) / np.sqrt(var + eps) * w + b


def erf_approx(x):
    """codec.rs:3890: Abramowitz & Stegun 7.1.26."""
    s = np.sign(x)
    s[s == 0] = 1.0
    a = np.abs(x)
    t = 1.0 / (1.0 + 0.3275911 * a)
    poly = (((((1.061405429 * t - 1.453152027) * t) + 1.421413741) * t - 0.284496736) * t + 0.254829592) * t
    return s * (1.0 - poly * np.exp(-a * a))


def gelu_erf(x):
    """codec.rs:3886."""
    return 0.5 * x * (1.0 + erf_approx(x * np.sqrt(0.5)))


def upsample_stage(x, w: CodecWeights, i):
    """codec.rs:3338 + 3438: transposed conv (k 2, stride 2), then a ConvNeXt
    block (depthwise causal conv 7, LayerNorm, 1024 -> 4096 GELU -> 1024,
    gamma, residual)."""
    p = f"quantizer.upsample.{i}"
    H, E = HIDDEN, CONVNEXT_EXPANDED
    y = conv_transpose_1d(x, w.get(f"{p}.0.conv.weight", [UPSAMPLE_FACTOR, H, H]), [UPSAMPLE_FACTOR, H, H],
                          w.get(f"{p}.0.conv.bias", [H]), UPSAMPLE_FACTOR)
    h = depthwise_causal_conv1d(y, w.get(f"{p}.1.dwconv.conv.weight", [CONVNEXT_KERNEL, 1, H]),
                                w.get(f"{p}.1.dwconv.conv.bias", [H]))
    h = layer_norm(h, w.get(f"{p}.1.norm.weight", [H]), w.get(f"{p}.1.norm.bias", [H]), CONVNEXT_EPS)
    h = gelu_erf(h @ w.get(f"{p}.1.pwconv1.weight", [H, E]).reshape(E, H).T + w.get(f"{p}.1.pwconv1.bias", [E]))
    h = h @ w.get(f"{p}.1.pwconv2.weight", [E, H]).reshape(H, E).T + w.get(f"{p}.1.pwconv2.bias", [H])
    return y + h * w.get(f"{p}.1.gamma", [H])


def rvq_decode_latents(lat, w: CodecWeights):
    """codec.rs:1282: post module, then the two upsample stages (x4 frames)."""
    x = post_module(lat, w)
    for i in range(UPSAMPLE_STAGES):
        x = upsample_stage(x, w, i)
    return x


# ---- decoder (codec.rs:1941-2293) ------------------------------------------

def snake(x, alpha):
    """codec.rs:2162 snake_activation_frame_major: x + sin(a x)^2 / a, |a| < 1e-8 -> 1e-8."""
    a = np.where(np.abs(alpha) < 1e-8, 1e-8, alpha)
    return x + np.sin(a * x) ** 2 / a


def round_f16(x):
    """tensor.rs round_f32_to_f16 of the float32 value (kept in x's dtype)."""
    return x.astype(np.float32).astype(np.float16).astype(x.dtype)


def causal_conv1d(x, weight, dims, bias, dilation=1):
    """codec.rs:2212 causal_conv_1d_frame_major at stride 1: left padding
    (kernel - 1) * dilation, the padded input rounded to f16, weight ggml
    [kernel, in, out]."""
    kernel, in_ch, out_ch = dims
    W = weight.reshape(out_ch, in_ch, kernel)
    F = x.shape[0]
    pad = (kernel - 1) * dilation
    xp = round_f16(np.concatenate([np.zeros((pad, in_ch), x.dtype), x]))
    y = np.tile(bias, (F, 1))
    for k in range(kernel):
        y += xp[k * dilation:k * dilation + F] @ W[:, :, k].T
    return y


def residual_unit(x, w: CodecWeights, p, C, dilation):
    """codec.rs:2085 forward_codec_residual_unit_impl."""
    b = snake(x, w.get(f"{p}.block.0.alpha", [1, C, 1]))
    b = causal_conv1d(b, w.get(f"{p}.block.1.conv.weight", [7, C, C]), [7, C, C], w.get(f"{p}.block.1.conv.bias", [C]),
                      dilation)
    b = snake(b, w.get(f"{p}.block.2.alpha", [1, C, 1]))
    b = causal_conv1d(b, w.get(f"{p}.block.3.conv.weight", [1, C, C]), [1, C, C], w.get(f"{p}.block.3.conv.bias", [C]))
    return x + b


def decoder_block(x, w: CodecWeights, i, C_in, stride):
    """codec.rs:2015 forward_codec_decoder_block."""
    p = f"decoder.model.{i}"
    C = DECODER_CHANNELS[i - 1]
    x = snake(x, w.get(f"{p}.block.0.alpha", [1, C_in, 1]))
    dims = w.t[f"{p}.block.1.conv.weight"][0] if f"{p}.block.1.conv.weight" in w.t else None
    if dims is None or len(dims) != 3 or dims[1:] != [C, C_in]:
        raise CodecOracleError(f"{p}.block.1.conv.weight: expected [k, {C}, {C_in}], got {dims}")
    x = conv_transpose_1d(x, w.get(f"{p}.block.1.conv.weight"), dims, w.get(f"{p}.block.1.conv.bias", [C]), stride)
    for u, d in zip((2, 3, 4), (1, 3, 9)):
        x = residual_unit(x, w, f"{p}.block.{u}", C, d)
    return x


def forward_codec_decoder(hidden, w: CodecWeights):
    """codec.rs:1941: entry conv 1024 -> 1536 (kernel 7), 4 blocks (x8, x8,
    x4, x2), snake, output conv 96 -> 1 (kernel 7), tanh."""
    x = causal_conv1d(hidden, w.get("decoder.model.0.conv.weight", [7, LATENT_DIM, DECODER_ENTRY_CHANNELS]),
                      [7, LATENT_DIM, DECODER_ENTRY_CHANNELS], w.get("decoder.model.0.conv.bias",
                                                                      [DECODER_ENTRY_CHANNELS]))
    C = DECODER_ENTRY_CHANNELS
    for i, r in enumerate(DECODER_RATES, start=1):
        x = decoder_block(x, w, i, C, r)
        C = DECODER_CHANNELS[i - 1]
    x = snake(x, w.get("decoder.model.5.alpha", [1, 96, 1]))
    x = causal_conv1d(x, w.get("decoder.model.6.conv.weight", [7, 96, 1]), [7, 96, 1],
                      w.get("decoder.model.6.conv.bias", [1]))
    return np.tanh(x[:, 0])


def decode_waveform(codes, num_codebooks, n_frames, w: CodecWeights):
    """codec.rs:1690: RVQ lookup -> latents -> decoder; mono PCM in [-1, 1]."""
    lat = rvq_lookup_codes(codes, num_codebooks, n_frames, w)
    return forward_codec_decoder(rvq_decode_latents(lat, w), w)


def pcm_to_wav(samples, sample_rate=SAMPLE_RATE):
    """wav.rs:7: 16-bit mono PCM, samples clamped to [-1, 1] and truncated
    toward zero after scaling by 32767."""
    s = np.clip(np.asarray(samples, np.float32), -1.0, 1.0)
    pcm = (s * np.float32(32767.0)).astype(np.int16)
    n = pcm.size
    hdr = b"RIFF" + struct.pack("<I", 44 + 2 * n) + b"WAVEfmt " + struct.pack(
        "<IHHIIHH", 16, 1, 1, sample_rate, sample_rate * 2, 2, 16) + b"data" + struct.pack("<I", 2 * n)
    return hdr + pcm.tobytes()


# ---- reference-audio encoder: PCM -> prompt codes (codec.rs:1056-1212, 1740-1940) ----

ENCODER_RATES = (2, 4, 8, 8)
ENCODER_CHANNELS = (64, 128, 256, 512, 1024)
ENCODER_WINDOW = 512
FRAME_LENGTH = 2048


def causal_conv1d_strided(x, weight, dims, bias, stride):
    """codec.rs:2212 causal_conv_1d_frame_major at dilation 1 and any stride:
    left padding kernel - stride, the extra right padding of
    extra_padding_for_conv1d (codec.rs:2191), the padded input rounded to f16."""
    kernel, in_ch, out_ch = dims
    W = weight.reshape(out_ch, in_ch, kernel)
    F = x.shape[0]
    pad = max(kernel - stride, 0)
    n = np.ceil(np.float32(F - kernel + pad) / np.float32(stride) + np.float32(1.0))
    ideal = max(int(n) - 1, 0) * stride + max(kernel - pad, 0)
    extra = max(ideal - F, 0)
    P = F + pad + extra
    xp = round_f16(np.concatenate([np.zeros((pad, in_ch), x.dtype), x, np.zeros((extra, in_ch), x.dtype)]))
    out = max(P - kernel, 0) // stride + 1
    y = np.tile(bias, (out, 1))
    for k in range(kernel):
        src = xp[k:k + (out - 1) * stride + 1:stride]
        y[:src.shape[0]] += src @ W[:, :, k].T
    return y


def pad_sample_count(n, frame_length=FRAME_LENGTH):
    """codec.rs:1926: up to a multiple of the frame length (one frame for no samples)."""
    return frame_length if n == 0 else (n + frame_length - 1) // frame_length * frame_length


def encoder_block(x, w: CodecWeights, i):
    """codec.rs:1740 forward_codec_encoder_block: residual units (dilations
    1, 3, 9), snake, strided down conv, and for the last block 4 transformer
    layers (window 512) + RMSNorm."""
    p = f"encoder.block.{i}.block"
    C, Co, s = ENCODER_CHANNELS[i - 1], ENCODER_CHANNELS[i], ENCODER_RATES[i - 1]
    for u, d in zip((0, 1, 2), (1, 3, 9)):
        x = residual_unit(x, w, f"{p}.{u}", C, d)
    x = snake(x, w.get(f"{p}.3.alpha", [1, C, 1]))
    k = w.t[f"{p}.4.conv.weight"][0][0] if f"{p}.4.conv.weight" in w.t else 2 * s
    x = causal_conv1d_strided(x, w.get(f"{p}.4.conv.weight", [k, C, Co]), [k, C, Co], w.get(f"{p}.4.conv.bias", [Co]),
                              s)
    if i == len(ENCODER_RATES):
        for layer in range(4):
            x = transformer_layer(x, w, layer, module=f"{p}.5", window=ENCODER_WINDOW)
        x = rms_norm(x, w.get(f"{p}.5.norm.weight", [HIDDEN]), NORM_EPS)
    return x


def forward_codec_encoder_frontend(audio, w: CodecWeights):
    """codec.rs:1104: pad to a multiple of 2,048 samples, entry conv 1 -> 64
    (kernel 7), 4 encoder blocks (/2, /4, /8, /8), snake, output conv
    1024 -> 1024 (kernel 3).  Returns (hidden [frames][1024], padded samples)."""
    audio = np.asarray(audio, np.float32).astype(w.dtype)
    n = pad_sample_count(audio.size)
    x = np.zeros((n, 1), w.dtype)
    x[:audio.size, 0] = audio
    x = causal_conv1d(x, w.get("encoder.block.0.conv.weight", [7, 1, 64]), [7, 1, 64],
                      w.get("encoder.block.0.conv.bias", [64]))
    for i in range(1, len(ENCODER_RATES) + 1):
        x = encoder_block(x, w, i)
    x = snake(x, w.get("encoder.block.5.alpha", [1, HIDDEN, 1]))
    x = causal_conv1d(x, w.get("encoder.block.6.conv.weight", [3, HIDDEN, HIDDEN]), [3, HIDDEN, HIDDEN],
                      w.get("encoder.block.6.conv.bias", [HIDDEN]))
    return x, n


def downsample_stage(x, w: CodecWeights, i):
    """codec.rs:3360: conv (kernel 2, stride 2), then the ConvNeXt block of codec.rs:3392."""
    p = f"quantizer.downsample.{i}"
    H, E = HIDDEN, CONVNEXT_EXPANDED
    if x.shape[0] < 2:
        raise CodecOracleError("codec downsample requires at least 2 frames")
    y = causal_conv1d_strided(x, w.get(f"{p}.0.conv.weight", [2, H, H]), [2, H, H], w.get(f"{p}.0.conv.bias", [H]),
                              2)
    if y.shape[0] != (x.shape[0] - 2) // 2 + 1:  # an odd frame count (codec.rs:3382, 3398)
        raise CodecOracleError("codec downsample convnext input length mismatch")
    h = depthwise_causal_conv1d(y, w.get(f"{p}.1.dwconv.conv.weight", [CONVNEXT_KERNEL, 1, H]),
                                w.get(f"{p}.1.dwconv.conv.bias", [H]))
    h = layer_norm(h, w.get(f"{p}.1.norm.weight", [H]), w.get(f"{p}.1.norm.bias", [H]), CONVNEXT_EPS)
    h = gelu_erf(h @ w.get(f"{p}.1.pwconv1.weight", [H, E]).reshape(E, H).T + w.get(f"{p}.1.pwconv1.bias", [E]))
    h = h @ w.get(f"{p}.1.pwconv2.weight", [E, H]).reshape(H, E).T + w.get(f"{p}.1.pwconv2.bias", [H])
    return y + h * w.get(f"{p}.1.gamma", [H])


def forward_codec_quantizer_encode_stage(x, w: CodecWeights):
    """codec.rs:1020: two downsample stages (/4 frames), the 8-layer pre
    module (window 128) and its RMSNorm."""
    for i in range(UPSAMPLE_STAGES):
        x = downsample_stage(x, w, i)
    for layer in range(LAYERS):
        x = transformer_layer(x, w, layer, module="quantizer.pre_module")
    return rms_norm(x, w.get("quantizer.pre_module.norm.weight", [HIDDEN]), NORM_EPS)


def rvq_encode_latents_nearest(lat, w: CodecWeights, margins=False):
    """codec.rs:2598 + nearest_code_for_residual (2453-2505): per frame and
    codebook in order, in_proj of the residual (+ bias), the codebook row of
    the largest cosine similarity (first on ties), residual -= that code's
    out_proj projection.  Returns (codes [10][frames], final residual L2
    [frames]) and, with margins, each choice's score gap to the runner-up."""
    F = lat.shape[0]
    codes = np.zeros((1 + RESIDUAL_QUANTIZERS, F), np.int64)
    gaps = np.zeros((1 + RESIDUAL_QUANTIZERS, F))
    res = lat.astype(w.dtype).copy()
    for cb in range(1 + RESIDUAL_QUANTIZERS):
        book, wo, bo = w.quantizer(cb)
        p = "quantizer.semantic_quantizer.quantizers.0" if cb == 0 else f"quantizer.quantizer.quantizers.{cb - 1}"
        wi = w.get(f"{p}.in_proj.weight", [1, HIDDEN, PROJ]).reshape(PROJ, HIDDEN)
        bi = w.get(f"{p}.in_proj.bias", [PROJ])
        proj = res @ wi.T + bi
        pn = np.sqrt(np.maximum((proj * proj).sum(axis=1, keepdims=True), 1e-12))
        rn = np.sqrt(np.maximum((book * book).sum(axis=1), 1e-12))
        score = (proj / pn) @ (book / rn[:, None]).T
        best = np.argmax(score, axis=1)
        codes[cb] = best
        srt = np.sort(score, axis=1)
        gaps[cb] = srt[:, -1] - srt[:, -2]
        res = res - (book[best] @ wo.T + bo)
    l2 = np.sqrt((res * res).sum(axis=1))
    return (codes, l2, gaps) if margins else (codes, l2)


def encode_reference_audio(audio, w: CodecWeights):
    """codec.rs:1056: encoder frontend, quantizer encode stage, nearest-code RVQ."""
    h, padded = forward_codec_encoder_frontend(audio, w)
    q = forward_codec_quantizer_encode_stage(h, w)
    codes, l2 = rvq_encode_latents_nearest(q, w)
    return codes, l2, h.shape[0], q.shape[0], padded
