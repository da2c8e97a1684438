"""Seeded synthetic codec GGUF files: the s2-pro codec's decode and
reference-audio encode tensors (fish-speech-codec architecture) with random
weights of the real shapes.

There is no network for the real checkpoint, so tests and the bench decode
codes through a file of the same layout: tensor names and ggml dims as the
reference loads them (crates/fish_s2_infer/src/codec.rs: quantizers
277-297 / 2356-2413, post module 496-540 / 822-910, upsample 414-447 /
721-820, decoder 1393-1440 / 1586-1679), all F16.  The decoder's transposed
convolutions take kernel 2 x stride, as in the DAC-style decoder the codec
uses (the reference reads the kernel from the weight's length,
codec.rs:2295).  Scales keep activations of order one through the stack.
"""
from __future__ import annotations

import os
import struct
from pathlib import Path

import numpy as np

HIDDEN, PROJ, FFN, EXPANDED = 1024, 8, 3072, 4096
LAYERS, UPSAMPLE_STAGES = 8, 2
ENTRY = 1536
RATES = (8, 8, 4, 2)
CHANNELS = (768, 384, 192, 96)
ENC_RATES = (2, 4, 8, 8)
ENC_CHANNELS = (64, 128, 256, 512, 1024)


def _layers(add, module, n):
    """The transformer layers of a codec module (codec.rs:315-333)."""
    for layer in range(n):
        p = f"{module}.layers.{layer}"
        add(f"{p}.attention.wqkv.weight", [HIDDEN, 3 * HIDDEN], HIDDEN ** -0.5)
        add(f"{p}.attention.wo.weight", [HIDDEN, HIDDEN], HIDDEN ** -0.5)
        add(f"{p}.attention_norm.weight", [HIDDEN], 0.1, 1.0)
        add(f"{p}.ffn_norm.weight", [HIDDEN], 0.1, 1.0)
        add(f"{p}.feed_forward.w1.weight", [HIDDEN, FFN], HIDDEN ** -0.5)
        add(f"{p}.feed_forward.w3.weight", [HIDDEN, FFN], HIDDEN ** -0.5)
        add(f"{p}.feed_forward.w2.weight", [FFN, HIDDEN], FFN ** -0.5)
        add(f"{p}.attention_layer_scale.gamma", [HIDDEN], 0.02, 0.1)
        add(f"{p}.ffn_layer_scale.gamma", [HIDDEN], 0.02, 0.1)


def _convnext(add, p):
    """The ConvNeXt block of an upsample or downsample stage (codec.rs:429-447)."""
    add(f"{p}.1.gamma", [HIDDEN], 0.02, 0.1)
    add(f"{p}.1.dwconv.conv.weight", [7, 1, HIDDEN], 7 ** -0.5)
    add(f"{p}.1.dwconv.conv.bias", [HIDDEN], 0.02)
    add(f"{p}.1.norm.weight", [HIDDEN], 0.1, 1.0)
    add(f"{p}.1.norm.bias", [HIDDEN], 0.02)
    add(f"{p}.1.pwconv1.weight", [HIDDEN, EXPANDED], HIDDEN ** -0.5)
    add(f"{p}.1.pwconv1.bias", [EXPANDED], 0.02)
    add(f"{p}.1.pwconv2.weight", [EXPANDED, HIDDEN], EXPANDED ** -0.5)
    add(f"{p}.1.pwconv2.bias", [HIDDEN], 0.02)


def _tensors():
    """(name, ggml dims, std, mean) of every tensor, in file order."""
    out = []

    def add(name, dims, std, mean=0.0):
        out.append((name, list(dims), std, mean))

    for cb in range(10):
        p = "quantizer.semantic_quantizer.quantizers.0" if cb == 0 else f"quantizer.quantizer.quantizers.{cb - 1}"
        n = 4096 if cb == 0 else 1024
        add(f"{p}.in_proj.weight", [1, HIDDEN, PROJ], HIDDEN ** -0.5)
        add(f"{p}.in_proj.bias", [PROJ], 0.02)
        add(f"{p}.out_proj.weight", [1, PROJ, HIDDEN], PROJ ** -0.5)
        add(f"{p}.out_proj.bias", [HIDDEN], 0.02)
        add(f"{p}.codebook.weight", [PROJ, n], 1.0)
    _layers(add, "quantizer.post_module", LAYERS)
    add("quantizer.post_module.norm.weight", [HIDDEN], 0.1, 1.0)
    for i in range(UPSAMPLE_STAGES):
        p = f"quantizer.upsample.{i}"
        add(f"{p}.0.conv.weight", [2, HIDDEN, HIDDEN], HIDDEN ** -0.5)
        add(f"{p}.0.conv.bias", [HIDDEN], 0.02)
        _convnext(add, p)
    # the reference-audio encoder (codec.rs:1323-1390, 1473-1584)
    add("encoder.block.0.conv.weight", [7, 1, 64], 7 ** -0.5)
    add("encoder.block.0.conv.bias", [64], 0.02)
    for i, (r, c) in enumerate(zip(ENC_RATES, ENC_CHANNELS[:-1]), start=1):
        p = f"encoder.block.{i}.block"
        co = ENC_CHANNELS[i]
        for u in range(3):
            q = f"{p}.{u}"
            add(f"{q}.block.0.alpha", [1, c, 1], 0.1, 1.0)
            add(f"{q}.block.1.conv.weight", [7, c, c], 0.7 * (7 * c) ** -0.5)
            add(f"{q}.block.1.conv.bias", [c], 0.02)
            add(f"{q}.block.2.alpha", [1, c, 1], 0.1, 1.0)
            add(f"{q}.block.3.conv.weight", [1, c, c], 0.5 * c ** -0.5)
            add(f"{q}.block.3.conv.bias", [c], 0.02)
        add(f"{p}.3.alpha", [1, c, 1], 0.1, 1.0)
        add(f"{p}.4.conv.weight", [2 * r, c, co], (2 * r * c) ** -0.5)
        add(f"{p}.4.conv.bias", [co], 0.02)
        if i == len(ENC_RATES):
            _layers(add, f"{p}.5", 4)
            add(f"{p}.5.norm.weight", [HIDDEN], 0.1, 1.0)
    add("encoder.block.5.alpha", [1, HIDDEN, 1], 0.1, 1.0)
    add("encoder.block.6.conv.weight", [3, HIDDEN, HIDDEN], (3 * HIDDEN) ** -0.5)
    add("encoder.block.6.conv.bias", [HIDDEN], 0.02)
    # the quantizer's encode side: downsample stages and pre module (codec.rs:357-391, 450-494)
    for i in range(UPSAMPLE_STAGES):
        p = f"quantizer.downsample.{i}"
        add(f"{p}.0.conv.weight", [2, HIDDEN, HIDDEN], (2 * HIDDEN) ** -0.5)
        add(f"{p}.0.conv.bias", [HIDDEN], 0.02)
        _convnext(add, p)
    _layers(add, "quantizer.pre_module", LAYERS)
    add("quantizer.pre_module.norm.weight", [HIDDEN], 0.1, 1.0)
    add("decoder.model.0.conv.weight", [7, HIDDEN, ENTRY], (7 * HIDDEN) ** -0.5)
    add("decoder.model.0.conv.bias", [ENTRY], 0.02)
    c_in = ENTRY
    for i, (r, c) in enumerate(zip(RATES, CHANNELS), start=1):
        p = f"decoder.model.{i}"
        add(f"{p}.block.0.alpha", [1, c_in, 1], 0.1, 1.0)
        add(f"{p}.block.1.conv.weight", [2 * r, c, c_in], (c_in * 2) ** -0.5)
        add(f"{p}.block.1.conv.bias", [c], 0.02)
        for u in (2, 3, 4):
            q = f"{p}.block.{u}"
            add(f"{q}.block.0.alpha", [1, c, 1], 0.1, 1.0)
            add(f"{q}.block.1.conv.weight", [7, c, c], 0.7 * (7 * c) ** -0.5)
            add(f"{q}.block.1.conv.bias", [c], 0.02)
            add(f"{q}.block.2.alpha", [1, c, 1], 0.1, 1.0)
            add(f"{q}.block.3.conv.weight", [1, c, c], 0.5 * c ** -0.5)
            add(f"{q}.block.3.conv.bias", [c], 0.02)
        c_in = c
    add("decoder.model.5.alpha", [1, 96, 1], 0.1, 1.0)
    add("decoder.model.6.conv.weight", [7, 96, 1], 0.2 * (7 * 96) ** -0.5)
    add("decoder.model.6.conv.bias", [1], 0.02)
    return out


def _gguf_string(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def write_codec_gguf(path: str | os.PathLike, seed: int = 1234) -> Path:
    """Write the synthetic codec file (about 770 MB) to `path`."""
    path = Path(path)
    specs = _tensors()
    rng = np.random.default_rng(seed)
    head = bytearray(b"GGUF")
    head += struct.pack("<IQQ", 3, len(specs), 2)
    head += _gguf_string("general.architecture") + struct.pack("<I", 8) + _gguf_string("fish-speech-codec")
    head += _gguf_string("general.alignment") + struct.pack("<II", 4, 32)
    offsets, off = [], 0
    for name, dims, _, _ in specs:
        n = int(np.prod(dims))
        offsets.append(off)
        head += _gguf_string(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims)
        head += struct.pack("<IQ", 1, off)
        off = (off + 2 * n + 31) // 32 * 32
    tmp = path.with_name(path.name + f".tmp{os.getpid()}")
    with open(tmp, "wb") as f:
        f.write(head)
        f.write(b"\0" * ((-len(head)) % 32))
        base = f.tell()
        for (name, dims, std, mean), o in zip(specs, offsets):
            n = int(np.prod(dims))
            v = (rng.standard_normal(n, dtype=np.float32) * np.float32(std) + np.float32(mean)).astype(np.float16)
            f.seek(base + o)
            f.write(v.tobytes())
        f.truncate(base + off)
    os.replace(tmp, path)
    return path


def cached_codec_gguf(directory: str | os.PathLike | None = None, seed: int = 1234) -> Path:
    """The synthetic codec file in `directory` (default: the model cache of
    synth.default_model_dir()), written on first use."""
    from .synth import default_model_dir
    d = Path(directory) if directory else default_model_dir()
    d.mkdir(parents=True, exist_ok=True)
    p = d / f"codec_synth_v2_{seed}.gguf"
    if not p.exists():
        write_codec_gguf(p, seed)
    return p
