"""Python mirror of the reference's `rust-pure` Dual-AR interface over libs2d.so.

Names, argument meaning and error behaviour follow crate fish_s2_infer
(paths relative to the reference repository root):

  SlowArState.open/prefill/step/reset/n_past/graph_spec   slow_ar.rs:372-528
  FastArWeights, forward_codebook_prefix,
  generate_codebooks_for_semantic                         fast_ar.rs:195-470
  generate_codes, GenerateParams, GenerateCodesResult     generate.rs:13-221
  SamplerParams, SeededRng, sample_token                  sampling.rs:12-241
  PromptTensor, transpose_to_time_major                   prompt.rs:59-103
  CudaMatmulBackend (the MatmulBackend op seam)           backend.rs:5-121

Every call runs on the GPU through the C ABI of include/s2d.h.  There is no
CPU fallback: loading fails loudly if libs2d.so is missing, and calls raise
S2dError (the counterpart of InferError::Message, error.rs:3-15) when the
library reports an error.
"""
from __future__ import annotations

import ctypes
import dataclasses
from pathlib import Path
from typing import Optional, Sequence

import numpy as np

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libs2d.so"

LOGITS_NONE, LOGITS_ALLOWED, LOGITS_FULL = 0, 1, 2
_LOGITS = {"none": LOGITS_NONE, "allowed": LOGITS_ALLOWED, "full": LOGITS_FULL}


class S2dError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class _Config(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int32), ("max_seq", ctypes.c_int32),
                ("max_batch", ctypes.c_int32), ("flags", ctypes.c_int32), ("kv_pages", ctypes.c_int32)]


_SPEC_INTS1 = ["slow_layers", "hidden", "ffn", "heads", "kv_heads", "head_dim", "context_length",
               "fast_layers", "fast_ffn", "fast_heads", "fast_kv_heads", "fast_head_dim",
               "fast_context_length"]
_SPEC_FLOATS = ["rope_base", "rms_eps", "fast_rope_base", "fast_rms_eps"]
_SPEC_INTS2 = ["codebook_size", "num_codebooks", "semantic_begin_id", "semantic_end_id",
               "vocab_size", "codebook_rows", "linear_type"]


class _Spec(ctypes.Structure):
    _fields_ = ([(n, ctypes.c_int32) for n in _SPEC_INTS1] +
                [(n, ctypes.c_float) for n in _SPEC_FLOATS] +
                [(n, ctypes.c_int32) for n in _SPEC_INTS2])


class _Sampler(ctypes.Structure):
    _fields_ = [("temperature", ctypes.c_float), ("top_p", ctypes.c_float),
                ("top_k", ctypes.c_int32)]


class _GenParams(ctypes.Structure):
    _fields_ = [("max_new_tokens", ctypes.c_uint32), ("temperature", ctypes.c_float),
                ("top_p", ctypes.c_float), ("top_k", ctypes.c_int32),
                ("min_tokens_before_end", ctypes.c_uint32), ("im_end_id", ctypes.c_uint32)]


class _TpShard(ctypes.Structure):
    _fields_ = [(f, ctypes.c_int32) for f in ("heads", "kv_heads", "head0", "kv_head0", "ffn", "ffn0")]


class _Profile(ctypes.Structure):
    _fields_ = [("prefill_ms", ctypes.c_double), ("decode_ms", ctypes.c_double),
                ("frames", ctypes.c_uint32), ("kernels_per_frame", ctypes.c_uint32),
                ("prefill_kernels", ctypes.c_uint32), ("frame_launches", ctypes.c_uint32)]


_P = ctypes.POINTER
_f32p = _P(ctypes.c_float)
_i32p = _P(ctypes.c_int32)
_u32p = _P(ctypes.c_uint32)
_u16p = _P(ctypes.c_uint16)
_u64p = _P(ctypes.c_uint64)

# symbol -> (restype, argtypes); every function declared in include/s2d.h
SIGNATURES = {
    "s2d_open": (ctypes.c_int32, [ctypes.c_char_p, _P(_Config), _P(ctypes.c_void_p),
                                  ctypes.c_char_p, ctypes.c_size_t]),
    "s2d_open_tp": (ctypes.c_int32, [ctypes.c_char_p, _P(_Config), ctypes.c_int32, ctypes.c_int32,
                                     ctypes.c_char_p, _P(ctypes.c_void_p), ctypes.c_char_p,
                                     ctypes.c_size_t]),
    "s2d_tp_plan": (ctypes.c_int32, [_P(_Spec), ctypes.c_int32, ctypes.c_int32, _P(_TpShard)]),
    "s2d_nccl_unique_id": (ctypes.c_int32, [ctypes.c_char_p, ctypes.c_size_t]),
    "s2d_close": (None, [ctypes.c_void_p]),
    "s2d_last_error": (ctypes.c_char_p, [ctypes.c_void_p]),
    "s2d_graph_spec": (ctypes.c_int32, [ctypes.c_void_p, _P(_Spec)]),
    "s2d_reset": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int32]),
    "s2d_n_past": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int32, _i32p]),
    "s2d_prefill": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int32, _i32p, ctypes.c_int64,
                                     _f32p, _f32p, ctypes.c_int32, ctypes.c_uint32]),
    "s2d_step": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int32, _i32p, ctypes.c_int64,
                                  _f32p, _f32p, ctypes.c_int32, ctypes.c_uint32]),
    "s2d_fast_prefix_logits": (ctypes.c_int32, [ctypes.c_void_p, _f32p, _u32p, ctypes.c_int64,
                                                _f32p]),
    "s2d_generate_codebooks": (ctypes.c_int32, [ctypes.c_void_p, _f32p, ctypes.c_uint32,
                                                _P(_Sampler), _u64p, _u32p]),
    "s2d_generate_codes": (ctypes.c_int32, [ctypes.c_void_p, _u32p, ctypes.c_int32, ctypes.c_int32,
                                            _P(_GenParams), _u64p, _i32p, _u32p, _P(_Profile)]),
    "s2d_generate_codes_batch": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int32,
                                                  _P(ctypes.c_void_p), _i32p, ctypes.c_int32,
                                                  _P(_GenParams), ctypes.c_int32, ctypes.c_uint64,
                                                  _u64p, _i32p, _u32p, _P(_Profile)]),
    "s2d_serve_begin": (ctypes.c_int32, [ctypes.c_void_p, _P(_GenParams), ctypes.c_int32, ctypes.c_uint64]),
    "s2d_serve_admit": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int32, _u32p, ctypes.c_int32, ctypes.c_int32,
                                         ctypes.c_uint64]),
    "s2d_serve_step": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int32, _i32p, _u32p]),
    "s2d_serve_collect": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int32, _i32p, _u32p, _u64p]),
    "s2d_serve_free_pages": (ctypes.c_int32, [ctypes.c_void_p, _i32p]),
    "s2d_philox4x32_10": (ctypes.c_int32, [_u32p, _u32p, _u32p]),
    "s2d_profile_batch": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int32, _P(ctypes.c_double),
                                           ctypes.c_int32]),
    "s2d_sample_token": (ctypes.c_int32, [ctypes.c_void_p, _f32p, ctypes.c_int64, _P(_Sampler),
                                          ctypes.c_int64, _u64p, _u32p]),
    "s2d_dequant_tensor": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_char_p, _f32p,
                                            ctypes.c_int64]),
    "s2d_profile_kernel": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                                            _P(ctypes.c_double), _P(ctypes.c_double)]),
    "s2d_profile_engine": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int32, _u64p, ctypes.c_int64,
                                            _i32p, _P(ctypes.c_double)]),
    "s2d_op_linear_f16": (ctypes.c_int32, [ctypes.c_void_p, _f32p, _u16p, ctypes.c_int64,
                                           ctypes.c_int64, _f32p]),
    "s2d_op_rows_linear_f16": (ctypes.c_int32, [ctypes.c_void_p, _f32p, ctypes.c_int64, ctypes.c_int64,
                                                _u16p, _u16p, ctypes.c_int64, _f32p, ctypes.c_int32,
                                                ctypes.c_int32, _f32p]),
    "s2d_op_prefill_attention": (ctypes.c_int32, [ctypes.c_void_p, _f32p, _u16p, _u16p, ctypes.c_int64,
                                                  ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                                  ctypes.c_int64, ctypes.c_int32, _f32p]),
    "s2d_op_batch_attention": (ctypes.c_int32, [ctypes.c_void_p, _f32p, _u16p, _u16p, ctypes.c_int64,
                                                ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                                _i32p, _i32p, ctypes.c_int32, ctypes.c_int32, _f32p]),
    "s2d_op_rms_norm": (ctypes.c_int32, [ctypes.c_void_p, _f32p, _f32p, ctypes.c_int64,
                                         ctypes.c_int64, ctypes.c_float, _f32p]),
    "s2d_op_rope_normal": (ctypes.c_int32, [ctypes.c_void_p, _f32p, ctypes.c_int64, ctypes.c_int64,
                                            ctypes.c_int64, ctypes.c_float, _f32p]),
    "s2d_op_gqa_decode_attention": (ctypes.c_int32, [ctypes.c_void_p, _f32p, _f32p, _f32p,
                                                     ctypes.c_int32, ctypes.c_int32,
                                                     ctypes.c_int32, ctypes.c_int32,
                                                     ctypes.c_float, _f32p]),
    "s2d_op_gqa_decode_attention_noalloc": (ctypes.c_int32, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
        ctypes.c_int32, ctypes.c_int32, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_char_p, ctypes.c_size_t]),
}

_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    """Load libs2d.so (built in-tree by fish_s2pro_b200.build)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m fish_s2pro_b200.build` "
                "(there is no CPU fallback)")
        l = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


def _ptr(a: np.ndarray, ct):
    return a.ctypes.data_as(_P(ct))


# ---------------------------------------------------------------------------
# data types (sampling.rs, generate.rs, prompt.rs, registry.rs)
# ---------------------------------------------------------------------------


@dataclasses.dataclass
class GraphSpec:
    slow_layers: int
    hidden: int
    ffn: int
    heads: int
    kv_heads: int
    head_dim: int
    context_length: int
    fast_layers: int
    fast_ffn: int
    fast_heads: int
    fast_kv_heads: int
    fast_head_dim: int
    fast_context_length: int
    rope_base: float
    rms_eps: float
    fast_rope_base: float
    fast_rms_eps: float
    codebook_size: int
    num_codebooks: int
    semantic_begin_id: int
    semantic_end_id: int
    vocab_size: int
    codebook_rows: int
    linear_type: int

    def codebook_input_dim(self) -> int:  # registry.rs:105-107
        return self.num_codebooks + 1


@dataclasses.dataclass
class SamplerParams:  # sampling.rs:12-27
    temperature: float = 0.7
    top_p: float = 0.7
    top_k: int = 30


@dataclasses.dataclass
class GenerateParams:  # generate.rs:13-32
    max_new_tokens: int = 512
    temperature: float = 0.7
    top_p: float = 0.7
    top_k: int = 30
    min_tokens_before_end: int = 64


class SeededRng:  # sampling.rs:35-52 (state advanced on the device)
    def __init__(self, seed: int):
        self.state = int(seed) & 0xFFFFFFFFFFFFFFFF


@dataclasses.dataclass
class PromptTensor:  # prompt.rs:59-67
    rows: int
    cols: int
    data: np.ndarray  # uint32, row-major rows x cols


def transpose_to_time_major(t: PromptTensor) -> np.ndarray:  # prompt.rs:77-103
    if t.rows == 0:
        raise S2dError(-1, "prompt rows must be non-zero")
    data = np.asarray(t.data, dtype=np.uint32).reshape(-1)
    if data.size != t.rows * t.cols:
        raise S2dError(-1, f"prompt data length mismatch: expected {t.rows * t.cols}, "
                           f"got {data.size}")
    if t.rows * t.cols and int(data.max()) > 0x7FFFFFFF:
        raise S2dError(-1, "prompt token id does not fit i32")
    return data.reshape(t.rows, t.cols).T.reshape(-1).astype(np.int32)


@dataclasses.dataclass
class SlowArStepResult:  # slow_ar.rs:242-246
    hidden: np.ndarray
    logits: Optional[np.ndarray]


@dataclasses.dataclass
class DecodeProfile:
    prefill_ms: float
    decode_ms: float
    frames: int
    kernels_per_frame: int
    prefill_kernels: int
    frame_launches: int


@dataclasses.dataclass
class GenerateCodesResult:  # generate.rs:39-46
    codes: np.ndarray  # int32, codebook-major num_codebooks x n_frames
    num_codebooks: int
    n_frames: int
    profile: DecodeProfile


# ---------------------------------------------------------------------------
# model handle
# ---------------------------------------------------------------------------


class SlowArState:
    """SlowArState (slow_ar.rs:372-528) backed by an sm_100a handle.  The
    handle also holds the Fast-AR weights (FastArWeights.from_state)."""

    def __init__(self, handle: ctypes.c_void_p, path: str):
        self._h = handle
        self.path = path
        spec = _Spec()
        self._check(lib().s2d_graph_spec(self._h, ctypes.byref(spec)))
        self._spec = GraphSpec(**{f: getattr(spec, f) for f, _ in _Spec._fields_})

    @classmethod
    def open(cls, transformer_path, max_seq_len: int = 32768, device: int = 0,
             max_batch: int = 1, tp: Optional[tuple] = None, kv_pages: int = 0) -> "SlowArState":
        """max_batch: sequences of generate_codes_batch or serving slots;
        kv_pages: pages of 64 positions in their shared KV pool (0: room for
        max_batch sequences of max_seq_len positions).  tp: (tp_size, tp_rank, nccl_id) to
        open one rank of a tensor-parallel Slow-AR (collective over the
        ranks; nccl_id from nccl_unique_id() on one rank)."""
        if max_seq_len <= 0:
            raise S2dError(-1, "max_seq_len must be non-zero")
        h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(1024)
        cfg = _Config(device=device, max_seq=max_seq_len, max_batch=max_batch, flags=0, kv_pages=kv_pages)
        if tp is not None and tp[0] > 1:
            size, rank, nid = tp
            rc = lib().s2d_open_tp(str(transformer_path).encode(), ctypes.byref(cfg), size, rank,
                                   bytes(nid), ctypes.byref(h), err, len(err))
        else:
            rc = lib().s2d_open(str(transformer_path).encode(), ctypes.byref(cfg), ctypes.byref(h),
                                err, len(err))
        if rc != 0:
            raise S2dError(rc, err.value.decode(errors="replace"))
        st = cls(h, str(transformer_path))
        st.max_batch = max(1, int(max_batch))
        return st

    def close(self) -> None:
        if self._h:
            lib().s2d_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def handle(self) -> ctypes.c_void_p:
        if not self._h:
            raise S2dError(-1, "state is closed")
        return self._h

    def _check(self, rc: int) -> None:
        if rc != 0:
            msg = lib().s2d_last_error(self._h)
            raise S2dError(rc, msg.decode(errors="replace") if msg else f"error {rc}")

    def graph_spec(self) -> GraphSpec:
        return self._spec

    def n_past(self) -> int:
        out = ctypes.c_int32()
        self._check(lib().s2d_n_past(self.handle, 0, ctypes.byref(out)))
        return int(out.value)

    def reset(self) -> None:
        self._check(lib().s2d_reset(self.handle, 0))

    def _eval(self, fn, flat: Sequence[int], logits: str, im_end_id: int) -> SlowArStepResult:
        toks = np.ascontiguousarray(np.asarray(flat, dtype=np.int32))
        hidden = np.empty(self._spec.hidden, dtype=np.float32)
        mode = _LOGITS[logits]
        lg = np.empty(self._spec.vocab_size, dtype=np.float32) if mode else None
        self._check(fn(self.handle, 0, _ptr(toks, ctypes.c_int32), toks.size,
                       _ptr(hidden, ctypes.c_float),
                       _ptr(lg, ctypes.c_float) if lg is not None else None, mode,
                       ctypes.c_uint32(im_end_id & 0xFFFFFFFF)))
        return SlowArStepResult(hidden=hidden, logits=lg)

    def prefill(self, flat_tokens, logits: str = "full", im_end_id: int = 0xFFFFFFFF):
        """slow_ar.rs:440-442.  logits: "full" (all vocab rows, like the
        reference), "allowed" (semantic rows + im_end_id, others -inf) or
        "none"."""
        return self._eval(lib().s2d_prefill, flat_tokens, logits, im_end_id)

    def step(self, flat_token, logits: str = "full", im_end_id: int = 0xFFFFFFFF):
        """slow_ar.rs:444-454."""
        return self._eval(lib().s2d_step, flat_token, logits, im_end_id)

    KERNELS = {"wqkv": 0, "wo": 1, "w13": 2, "w2": 3, "lm_head": 4}

    def profile_kernel(self, kernel: str, iters: int = 72) -> tuple:
        """(mean ms per launch, algorithmic bytes per launch) of one decode
        kernel on the resident weights (s2d_profile_kernel)."""
        ms, nb = ctypes.c_double(), ctypes.c_double()
        self._check(lib().s2d_profile_kernel(self.handle, self.KERNELS[kernel], iters,
                                             ctypes.byref(ms), ctypes.byref(nb)))
        return float(ms.value), float(nb.value)

    def profile_engine(self, program: int = 0, trace: bool = True, per_cta: bool = False):
        """Run one persistent-engine program once (s2d_profile_engine):
        0 the Slow-AR step, k >= 1 Fast-AR pass k, -1 the frame's whole
        Fast-AR.
        Returns (ms, trace) with trace shaped [2 CTAs][n_ops][4] in ns; with
        per_cta, (ms, trace, finish) where finish is [n_ops][CTAs] in ns."""
        n = ctypes.c_int32()
        ms = ctypes.c_double()
        buf = np.zeros(264 * 256, dtype=np.uint64) if trace else None
        self._check(lib().s2d_profile_engine(self.handle, program,
                                             _ptr(buf, ctypes.c_uint64) if trace else None,
                                             buf.size if trace else 0, ctypes.byref(n),
                                             ctypes.byref(ms)))
        tr = buf[: n.value * 8].reshape(2, n.value, 4) if trace else None
        if not per_cta:
            return float(ms.value), tr
        g = (int(np.count_nonzero(buf[n.value * 8:])) + n.value - 1) // max(n.value, 1) if trace else 0
        fin = buf[n.value * 8: n.value * (8 + g)].reshape(n.value, g) if trace else None
        return float(ms.value), tr, fin

    PROFILE_BATCH_KEYS = ("split", "gemm", "combine", "rope", "attention", "sample", "other", "total")

    def profile_batch(self, n_seq: int) -> dict:
        """ms of one batched frame per kernel category (s2d_profile_batch),
        after generate_codes_batch."""
        out = (ctypes.c_double * len(self.PROFILE_BATCH_KEYS))()
        self._check(lib().s2d_profile_batch(self._h, n_seq, out, len(out)))
        return dict(zip(self.PROFILE_BATCH_KEYS, list(out)))

    def dequant_tensor(self, name: str, count: int) -> np.ndarray:
        out = np.empty(count, dtype=np.float32)
        self._check(lib().s2d_dequant_tensor(self.handle, name.encode(), _ptr(out, ctypes.c_float),
                                             count))
        return out


class FastArWeights:
    """FastArWeights (fast_ar.rs:195-224): the Fast-AR layers are resident in
    the same device handle as the Slow-AR."""

    def __init__(self, state: SlowArState):
        self.state = state

    @classmethod
    def from_state(cls, state: SlowArState) -> "FastArWeights":
        return cls(state)


def forward_codebook_prefix(slow_hidden, prefix_codes, graph: GraphSpec,
                            weights: FastArWeights) -> np.ndarray:
    """fast_ar.rs:360-437."""
    st = weights.state
    h = np.ascontiguousarray(np.asarray(slow_hidden, dtype=np.float32))
    if h.size != graph.hidden:
        raise S2dError(-1, f"slow hidden size mismatch: expected {graph.hidden}, got {h.size}")
    pre = np.ascontiguousarray(np.asarray(prefix_codes, dtype=np.uint32))
    out = np.empty(graph.codebook_size, dtype=np.float32)
    st._check(lib().s2d_fast_prefix_logits(st.handle, _ptr(h, ctypes.c_float),
                                           _ptr(pre, ctypes.c_uint32) if pre.size else None,
                                           pre.size, _ptr(out, ctypes.c_float)))
    return out


def generate_codebooks_for_semantic(slow_hidden, semantic_code: int, graph: GraphSpec,
                                    weights: FastArWeights, sampler: SamplerParams,
                                    rng: SeededRng) -> list:
    """fast_ar.rs:440-470."""
    st = weights.state
    h = np.ascontiguousarray(np.asarray(slow_hidden, dtype=np.float32))
    out = np.empty(graph.num_codebooks, dtype=np.uint32)
    sp = _Sampler(sampler.temperature, sampler.top_p, sampler.top_k)
    state = ctypes.c_uint64(rng.state)
    st._check(lib().s2d_generate_codebooks(st.handle, _ptr(h, ctypes.c_float), semantic_code,
                                           ctypes.byref(sp), ctypes.byref(state),
                                           _ptr(out, ctypes.c_uint32)))
    rng.state = state.value
    return [int(x) for x in out]


def sample_token(state: SlowArState, logits, params: SamplerParams,
                 always_include_id: Optional[int], rng: SeededRng) -> int:
    """sampling.rs:121-200 on the device sampler (at most 8192 logits)."""
    lg = np.ascontiguousarray(np.asarray(logits, dtype=np.float32))
    sp = _Sampler(params.temperature, params.top_p, params.top_k)
    s = ctypes.c_uint64(rng.state)
    out = ctypes.c_uint32()
    state._check(lib().s2d_sample_token(state.handle, _ptr(lg, ctypes.c_float), lg.size,
                                        ctypes.byref(sp),
                                        -1 if always_include_id is None else int(always_include_id),
                                        ctypes.byref(s), ctypes.byref(out)))
    rng.state = s.value
    return int(out.value)


def generate_codes(state: SlowArState, tokenizer, graph: GraphSpec, prompt: PromptTensor,
                   params: GenerateParams, fast_weights: FastArWeights,
                   rng: SeededRng) -> GenerateCodesResult:
    """generate.rs:117-221.  `tokenizer` is the S2TokenizerConfig (anything
    with an `im_end_id`) or the im_end id itself."""
    im_end = int(getattr(tokenizer, "im_end_id", tokenizer))
    data = np.ascontiguousarray(np.asarray(prompt.data, dtype=np.uint32).reshape(-1))
    if data.size != prompt.rows * prompt.cols:
        raise S2dError(-1, "prompt data length mismatch")
    k = max(graph.num_codebooks, 1)
    codes = np.zeros(k * max(params.max_new_tokens, 1), dtype=np.int32)
    gp = _GenParams(params.max_new_tokens, params.temperature, params.top_p, params.top_k,
                    params.min_tokens_before_end, im_end)
    s = ctypes.c_uint64(rng.state)
    n_frames = ctypes.c_uint32()
    prof = _Profile()
    state._check(lib().s2d_generate_codes(state.handle, _ptr(data, ctypes.c_uint32), prompt.rows,
                                          prompt.cols, ctypes.byref(gp), ctypes.byref(s),
                                          _ptr(codes, ctypes.c_int32), ctypes.byref(n_frames),
                                          ctypes.byref(prof)))
    rng.state = s.value
    n = int(n_frames.value)
    return GenerateCodesResult(
        codes=codes[: k * n].copy(), num_codebooks=k, n_frames=n,
        profile=DecodeProfile(prof.prefill_ms, prof.decode_ms, prof.frames,
                              prof.kernels_per_frame, prof.prefill_kernels,
                              prof.frame_launches))


def nccl_unique_id() -> bytes:
    """A fresh NCCL unique id for SlowArState.open(tp=...)."""
    buf = ctypes.create_string_buffer(128)
    rc = lib().s2d_nccl_unique_id(buf, len(buf))
    if rc != 0:
        raise S2dError(rc, "ncclGetUniqueId failed")
    return buf.raw


def tp_plan(spec: GraphSpec, tp_size: int, tp_rank: int) -> dict:
    """Rank tp_rank's shard of the Slow-AR under tp_size-way tensor
    parallelism (s2d_tp_plan): its query / KV heads and FFN columns."""
    c = _Spec(**{f: getattr(spec, f) for f, _ in _Spec._fields_})
    out = _TpShard()
    rc = lib().s2d_tp_plan(ctypes.byref(c), tp_size, tp_rank, ctypes.byref(out))
    if rc != 0:
        raise S2dError(rc, f"no {tp_size}-way split of this model")
    return {f: getattr(out, f) for f, _ in _TpShard._fields_}


RNG_SEEDED = 0  # the reference's SeededRng per sequence
RNG_PHILOX = 1  # Philox4x32-10, counter (draw index, sequence)


def generate_codes_batch(state: SlowArState, tokenizer, graph: GraphSpec,
                         prompts: Sequence[PromptTensor], params: GenerateParams,
                         fast_weights: FastArWeights, rngs: Sequence[SeededRng],
                         rng_kind: int = RNG_SEEDED, philox_key: int = 0):
    """generate_codes (generate.rs:117-221) over independent prompts at once,
    one result per prompt.  With RNG_SEEDED, rngs[i] is sequence i's
    SeededRng; with RNG_PHILOX its state is sequence i's draw counter.  The
    handle must have been opened with max_batch >= len(prompts)."""
    im_end = int(getattr(tokenizer, "im_end_id", tokenizer))
    n = len(prompts)
    if n != len(rngs):
        raise S2dError(-1, "one rng per prompt")
    rows = {p.rows for p in prompts}
    if len(rows) != 1:
        raise S2dError(-1, "prompts must share the row count (num_codebooks+1)")
    datas = []
    for p in prompts:
        d = np.ascontiguousarray(np.asarray(p.data, dtype=np.uint32).reshape(-1))
        if d.size != p.rows * p.cols:
            raise S2dError(-1, "prompt data length mismatch")
        datas.append(d)
    ptrs = (ctypes.c_void_p * n)(*[d.ctypes.data for d in datas])
    cols = np.array([p.cols for p in prompts], dtype=np.int32)
    k = max(graph.num_codebooks, 1)
    stride = k * max(params.max_new_tokens, 1)
    codes = np.zeros(n * stride, dtype=np.int32)
    frames = np.zeros(n, dtype=np.uint32)
    states = np.array([r.state for r in rngs], dtype=np.uint64)
    gp = _GenParams(params.max_new_tokens, params.temperature, params.top_p, params.top_k,
                    params.min_tokens_before_end, im_end)
    prof = _Profile()
    state._check(lib().s2d_generate_codes_batch(
        state.handle, n, ptrs, _ptr(cols, ctypes.c_int32), rows.pop(), ctypes.byref(gp),
        rng_kind, ctypes.c_uint64(philox_key), _ptr(states, ctypes.c_uint64),
        _ptr(codes, ctypes.c_int32), _ptr(frames, ctypes.c_uint32), ctypes.byref(prof)))
    out = []
    for i in range(n):
        rngs[i].state = int(states[i])
        f = int(frames[i])
        out.append(GenerateCodesResult(
            codes=codes[i * stride: i * stride + k * f].copy(), num_codebooks=k, n_frames=f,
            profile=DecodeProfile(prof.prefill_ms, prof.decode_ms, prof.frames,
                                  prof.kernels_per_frame, prof.prefill_kernels,
                                  prof.frame_launches)))
    return out


# ---------------------------------------------------------------------------
# op-level seam (MatmulBackend, backend.rs:5-121)
# ---------------------------------------------------------------------------


class CudaMatmulBackend:
    """The reference's MatmulBackend trait on the device.  Host arrays in and
    out; `state` may be None (default device, temporary buffers)."""

    def __init__(self, state: Optional[SlowArState] = None):
        self.state = state

    def name(self) -> str:
        return "cuda-sm100a"

    def _h(self):
        return self.state.handle if self.state is not None else None

    def _check(self, rc: int) -> None:
        if rc != 0:
            msg = lib().s2d_last_error(self._h()) if self.state is not None else b""
            raise S2dError(rc, (msg or b"").decode() or f"op failed ({rc})")

    def linear_f16(self, input, weight_f16_bits, input_dim: int, output_dim: int) -> np.ndarray:
        x = np.ascontiguousarray(np.asarray(input, dtype=np.float32))
        w = np.ascontiguousarray(np.asarray(weight_f16_bits, dtype=np.uint16))
        if x.size != input_dim:
            raise S2dError(-1, f"linear input length mismatch: expected {input_dim}, got {x.size}")
        if w.size != input_dim * output_dim:
            raise S2dError(-1, f"linear weight length mismatch: expected "
                               f"{input_dim * output_dim}, got {w.size}")
        out = np.empty(output_dim, dtype=np.float32)
        self._check(lib().s2d_op_linear_f16(self._h(), _ptr(x, ctypes.c_float),
                                            _ptr(w, ctypes.c_uint16), input_dim, output_dim,
                                            _ptr(out, ctypes.c_float)))
        return out

    def rms_norm_heads(self, input, weight, head_dim: int, eps: float) -> np.ndarray:
        x = np.ascontiguousarray(np.asarray(input, dtype=np.float32))
        w = np.ascontiguousarray(np.asarray(weight, dtype=np.float32))
        if x.size == 0:
            raise S2dError(-1, "rms_norm input is empty")
        if x.size % head_dim:
            raise S2dError(-1, f"head RMSNorm input length {x.size} is not a multiple of "
                               f"head_dim {head_dim}")
        out = np.empty_like(x)
        self._check(lib().s2d_op_rms_norm(self._h(), _ptr(x, ctypes.c_float),
                                          _ptr(w, ctypes.c_float), x.size, head_dim, eps,
                                          _ptr(out, ctypes.c_float)))
        return out

    def rms_norm(self, input, weight, eps: float) -> np.ndarray:
        x = np.asarray(input, dtype=np.float32)
        if x.size != np.asarray(weight).size:
            raise S2dError(-1, f"rms_norm length mismatch: input={x.size}, "
                               f"weight={np.asarray(weight).size}")
        return self.rms_norm_heads(x, weight, x.size, eps)

    def apply_rope_normal(self, values, head_dim: int, position: int, base: float) -> np.ndarray:
        """apply_rope_normal (attention.rs:172-206) over every head of values."""
        x = np.ascontiguousarray(np.asarray(values, dtype=np.float32))
        if x.size == 0 or x.size % head_dim:
            raise S2dError(-1, f"rope input length {x.size} is not a multiple of head_dim {head_dim}")
        out = np.empty_like(x)
        self._check(lib().s2d_op_rope_normal(self._h(), _ptr(x, ctypes.c_float), x.size, head_dim,
                                             position, base, _ptr(out, ctypes.c_float)))
        return out

    def gqa_decode_attention(self, query, keys, values, head_count: int, head_count_kv: int,
                             head_dim: int, token_count: int, attn_scale: float) -> np.ndarray:
        q = np.ascontiguousarray(np.asarray(query, dtype=np.float32))
        k = np.ascontiguousarray(np.asarray(keys, dtype=np.float32))
        v = np.ascontiguousarray(np.asarray(values, dtype=np.float32))
        out = np.empty(head_count * head_dim, dtype=np.float32)
        self._check(lib().s2d_op_gqa_decode_attention(
            self._h(), _ptr(q, ctypes.c_float), _ptr(k, ctypes.c_float), _ptr(v, ctypes.c_float),
            head_count, head_count_kv, head_dim, token_count, attn_scale,
            _ptr(out, ctypes.c_float)))
        return out
