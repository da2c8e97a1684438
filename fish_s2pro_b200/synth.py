"""Seeded synthetic fish-speech transformer GGUF files (see csrc/synth_gguf.c)."""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

from .configs import ModelConfig


class _SynthConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "slow_layers", "d", "heads", "kv_heads", "head_dim", "ffn", "vocab", "sem_begin",
        "sem_end", "fast_layers", "fast_heads", "fast_kv_heads", "fast_head_dim", "fast_ffn",
        "num_codebooks", "codebook_size", "context_length", "fast_context_length",
        "linear_type")] + [("rope_base", ctypes.c_float), ("eps", ctypes.c_float),
                            ("weight_std", ctypes.c_float), ("seed", ctypes.c_uint64)]


_libs: dict = {}


def _load(lib_path: str | os.PathLike | None = None):
    """The writer library: the package's libs2d_synth.so, or another build of
    csrc/synth_gguf.c at `lib_path` (the CPU reference arm of bench.py uses
    the oracle's build, so that its process maps no library of this
    package)."""
    key = str(lib_path) if lib_path else ""
    if key not in _libs:
        if lib_path is None:
            from . import build
            lib_path = build.build_synth()
        lib = ctypes.CDLL(str(lib_path))
        lib.s2d_synth_write_gguf.argtypes = [ctypes.c_char_p, ctypes.POINTER(_SynthConfig),
                                             ctypes.c_char_p, ctypes.c_size_t]
        lib.s2d_synth_write_gguf.restype = ctypes.c_int
        _libs[key] = lib
    return _libs[key]


def write_gguf(path: str | os.PathLike, m: ModelConfig,
               lib_path: str | os.PathLike | None = None) -> Path:
    """Write model `m` to `path` (overwritten).  Deterministic in m.seed."""
    lib = _load(lib_path)
    c = _SynthConfig(
        slow_layers=m.slow_layers, d=m.d, heads=m.heads, kv_heads=m.kv_heads,
        head_dim=m.head_dim, ffn=m.ffn, vocab=m.vocab, sem_begin=m.sem_begin, sem_end=m.sem_end,
        fast_layers=m.fast_layers, fast_heads=m.fast_heads, fast_kv_heads=m.fast_kv_heads,
        fast_head_dim=m.fast_head_dim, fast_ffn=m.fast_ffn, num_codebooks=m.num_codebooks,
        codebook_size=m.codebook_size, context_length=m.context_length,
        fast_context_length=m.fast_context_length, linear_type=m.linear_type,
        rope_base=m.rope_base, eps=m.eps, weight_std=m.weight_std, seed=m.seed)
    err = ctypes.create_string_buffer(512)
    p = Path(path)
    rc = lib.s2d_synth_write_gguf(str(p).encode(), ctypes.byref(c), err, len(err))
    if rc != 0:
        raise OSError(err.value.decode())
    return p


def default_model_dir() -> Path:
    """$S2D_MODEL_CACHE, else /dev/shm when it has room for a full-size model
    (a RAM-backed file makes the one-time upload faster), else /tmp."""
    env = os.environ.get("S2D_MODEL_CACHE")
    if env:
        return Path(env)
    try:
        st = os.statvfs("/dev/shm")
        if st.f_bavail * st.f_frsize > 40 << 30:
            return Path("/dev/shm/s2d_models")
    except OSError:
        pass
    return Path("/tmp/s2d_models")


def model_file_name(m: ModelConfig) -> str:
    return (f"{m.name}-L{m.slow_layers}F{m.fast_layers}-t{m.linear_type}-s{m.seed}"
            f"-d{m.d}-v{m.vocab}.gguf")


def cached_gguf(m: ModelConfig, directory: str | os.PathLike | None = None,
                lib_path: str | os.PathLike | None = None) -> Path:
    """Path of model `m` under `directory` (default: default_model_dir()),
    written on first use (with the writer at `lib_path`, see _load)."""
    d = Path(directory or default_model_dir())
    d.mkdir(parents=True, exist_ok=True)
    p = d / model_file_name(m)
    if not p.exists():
        tmp = p.with_suffix(f".tmp{os.getpid()}")
        write_gguf(tmp, m, lib_path)
        os.replace(tmp, p)
    return p
