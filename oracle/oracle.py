"""ctypes wrapper of the CPU oracle (libs2_oracle.so).

TEST INFRASTRUCTURE ONLY: the parity checker for the sm_100a path and the
timed CPU baseline.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
legs use it; nothing in fish_s2pro_b200 imports it.  Each function mirrors
the reference function named in oracle/s2_oracle.h.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path
from typing import Optional

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libs2_oracle.so"

_P = ctypes.POINTER
_f32p = _P(ctypes.c_float)
_i32p = _P(ctypes.c_int32)
_u32p = _P(ctypes.c_uint32)
_u16p = _P(ctypes.c_uint16)
_u64p = _P(ctypes.c_uint64)
_i64 = ctypes.c_int64


class OracleError(RuntimeError):
    pass


class GraphSpec(ctypes.Structure):
    _fields_ = ([(n, ctypes.c_int32) for n in (
        "slow_context_length", "slow_embedding_length", "slow_feed_forward_length",
        "slow_block_count", "slow_head_count", "slow_head_count_kv", "slow_head_dim")] +
        [("slow_rope_freq_base", ctypes.c_float), ("slow_rms_norm_eps", ctypes.c_float),
         ("slow_attention_qk_norm", ctypes.c_int32)] +
        [(n, ctypes.c_int32) for n in (
            "fast_context_length", "fast_embedding_length", "fast_feed_forward_length",
            "fast_block_count", "fast_head_count", "fast_head_count_kv", "fast_head_dim")] +
        [("fast_rope_freq_base", ctypes.c_float), ("fast_rms_norm_eps", ctypes.c_float),
         ("fast_attention_qk_norm", ctypes.c_int32)] +
        [(n, ctypes.c_int32) for n in (
            "codebook_size", "num_codebooks", "semantic_begin_id", "semantic_end_id",
            "scale_codebook_embeddings", "tie_word_embeddings", "fast_project_in")] +
        [("vocab_size", ctypes.c_int64), ("codebook_rows", ctypes.c_int64),
         ("fast_vocab_size", ctypes.c_int64)])


class GenParams(ctypes.Structure):
    _fields_ = [("max_new_tokens", ctypes.c_uint32), ("temperature", ctypes.c_float),
                ("top_p", ctypes.c_float), ("top_k", ctypes.c_int32),
                ("min_tokens_before_end", ctypes.c_uint32), ("im_end_id", ctypes.c_uint32)]


class LayerShape(ctypes.Structure):
    _fields_ = [("hidden_size", _i64), ("feed_forward_size", _i64), ("head_count", _i64),
                ("head_count_kv", _i64), ("head_dim", _i64), ("rope_base", ctypes.c_float),
                ("rms_norm_eps", ctypes.c_float)]


_W_NAMES = ["attention_norm", "q_norm", "k_norm", "wqkv", "wo", "ffn_norm", "w1", "w2", "w3"]


class LayerWeights(ctypes.Structure):
    _fields_ = [(n, _f32p) for n in _W_NAMES] + [("n_" + n, _i64) for n in _W_NAMES]


_T_NAMES = ["normalized", "query", "key", "value", "attention", "projected", "attn_hidden",
            "ffn_normalized", "gate", "up", "activated", "ffn_projected", "hidden"]


class LayerTrace(ctypes.Structure):
    _fields_ = [(n, _f32p) for n in _T_NAMES]


_SIGS = {
    "s2o_last_error": (ctypes.c_char_p, []),
    "s2o_f16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
    "s2o_f32_to_f16": (ctypes.c_uint16, [ctypes.c_float]),
    "s2o_round_f32_to_f16": (ctypes.c_float, [ctypes.c_float]),
    "s2o_rms_norm": (ctypes.c_int, [_f32p, _f32p, _i64, ctypes.c_float, _f32p]),
    "s2o_rms_norm_heads": (ctypes.c_int, [_f32p, _f32p, _i64, _i64, ctypes.c_float, _f32p]),
    "s2o_linear": (ctypes.c_int, [_f32p, _f32p, _i64, _i64, _f32p]),
    "s2o_matvec_f16": (ctypes.c_int, [_f32p, _u16p, _i64, _i64, _f32p]),
    "s2o_rope_normal": (ctypes.c_int, [_f32p, _i64, _i64, _i64, ctypes.c_float]),
    "s2o_gqa_decode_attention": (ctypes.c_int, [_f32p, _f32p, _f32p, _i64, _i64, _i64, _i64,
                                                ctypes.c_float, _f32p]),
    "s2o_swiglu_slow": (ctypes.c_int, [_f32p, _f32p, _i64, _f32p]),
    "s2o_swiglu_fast": (ctypes.c_int, [_f32p, _f32p, _i64, _f32p]),
    "s2o_rng_next_unit": (ctypes.c_double, [_u64p]),
    "s2o_build_semantic_bias": (ctypes.c_int, [_i64, ctypes.c_uint32, ctypes.c_uint32, _i64,
                                               _f32p]),
    "s2o_apply_semantic_bias": (ctypes.c_int, [_f32p, _f32p, _i64, ctypes.c_int, _i64]),
    "s2o_semantic_mask_logits": (ctypes.c_int, [_f32p, _i64, ctypes.c_uint32, ctypes.c_uint32,
                                                _i64, ctypes.c_int]),
    "s2o_sample_token": (ctypes.c_int, [_f32p, _i64, ctypes.c_float, ctypes.c_float,
                                        ctypes.c_int32, _i64, _u64p, _u32p]),
    "s2o_kv_new": (ctypes.c_void_p, [_i64, _i64, _i64, _i64]),
    "s2o_kv_free": (None, [ctypes.c_void_p]),
    "s2o_kv_write_token": (ctypes.c_int, [ctypes.c_void_p, _i64, _i64, _f32p, _f32p]),
    "s2o_kv_read_token": (ctypes.c_int, [ctypes.c_void_p, _i64, _i64, _f32p, _f32p]),
    "s2o_kv_decode_attention": (ctypes.c_int, [ctypes.c_void_p, _i64, _i64, _f32p, _i64,
                                               ctypes.c_float, _f32p]),
    "s2o_layer_forward": (ctypes.c_int, [_P(LayerShape), _P(LayerWeights), _f32p, _i64,
                                         ctypes.c_void_p, _i64, _i64, ctypes.c_int,
                                         _P(LayerTrace), _f32p]),
    "s2o_open": (ctypes.c_void_p, [ctypes.c_char_p, _i64, ctypes.c_int]),
    "s2o_close": (None, [ctypes.c_void_p]),
    "s2o_graph_spec": (ctypes.c_int, [ctypes.c_void_p, _P(GraphSpec)]),
    "s2o_set_threads": (ctypes.c_int, [ctypes.c_int]),
    "s2o_get_threads": (ctypes.c_int, []),
    "s2o_reset": (None, [ctypes.c_void_p]),
    "s2o_n_past": (_i64, [ctypes.c_void_p]),
    "s2o_eval": (ctypes.c_int, [ctypes.c_void_p, _i32p, _i64, _f32p, _f32p, ctypes.c_int, _i64]),
    "s2o_fast_prefix_logits": (ctypes.c_int, [ctypes.c_void_p, _f32p, _u32p, _i64, _f32p]),
    "s2o_generate_codebooks": (ctypes.c_int, [ctypes.c_void_p, _f32p, ctypes.c_uint32,
                                              ctypes.c_float, ctypes.c_float, ctypes.c_int32,
                                              _u64p, _u32p]),
    "s2o_generate_codes": (ctypes.c_int, [ctypes.c_void_p, _u32p, _i64, _i64, _P(GenParams),
                                          _u64p, _i32p, _u32p, _u32p]),
    "s2o_transpose_to_time_major": (ctypes.c_int, [_u32p, _i64, _i64, _i32p]),
    "s2o_compact_codes": (ctypes.c_int, [_i32p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                         _P(_i64)]),
    "s2o_gguf_open": (ctypes.c_void_p, [ctypes.c_char_p]),
    "s2o_gguf_close": (None, [ctypes.c_void_p]),
    "s2o_gguf_tensor_count": (_i64, [ctypes.c_void_p]),
    "s2o_gguf_version": (ctypes.c_uint32, [ctypes.c_void_p]),
    "s2o_gguf_data_start": (ctypes.c_uint64, [ctypes.c_void_p]),
    "s2o_gguf_tensor_info": (ctypes.c_int, [ctypes.c_void_p, _i64, _P(ctypes.c_char_p),
                                            _P(ctypes.c_int32), _P(ctypes.c_uint64), _u32p,
                                            _P(ctypes.c_uint64), _P(ctypes.c_uint64)]),
    "s2o_gguf_tensor_data": (ctypes.c_void_p, [ctypes.c_void_p, ctypes.c_char_p,
                                               _P(ctypes.c_uint64)]),
    "s2o_gguf_metadata": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_char_p,
                                         ctypes.c_size_t]),
    "s2o_dequant_row": (ctypes.c_int, [ctypes.c_uint32, ctypes.c_void_p, _i64, _f32p]),
    "s2o_ggml_byte_len": (_i64, [ctypes.c_uint32, _i64]),
}

_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        src = HERE / "s2_oracle.c"
        if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
            subprocess.run(["make", "-C", str(HERE)], check=True, capture_output=True)
        l = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


def _f(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _p(a, ct=ctypes.c_float):
    return None if a is None else a.ctypes.data_as(_P(ct))


def _check(rc: int) -> None:
    if rc != 0:
        raise OracleError(lib().s2o_last_error().decode(errors="replace"))


# ---- scalar / op level ----------------------------------------------------

def f16_to_f32(bits: int) -> float:
    return lib().s2o_f16_to_f32(bits)


def f32_to_f16(v: float) -> int:
    return lib().s2o_f32_to_f16(v)


def round_f32_to_f16(v: float) -> float:
    return lib().s2o_round_f32_to_f16(v)


def rms_norm(x, w, eps):
    x, w = _f(x), _f(w)
    if x.size == 0:
        raise OracleError("rms_norm input is empty")
    if x.size != w.size:
        raise OracleError(f"rms_norm length mismatch: input={x.size}, weight={w.size}")
    out = np.empty_like(x)
    _check(lib().s2o_rms_norm(_p(x), _p(w), x.size, eps, _p(out)))
    return out


def rms_norm_heads(x, w, head_dim, eps):
    x, w = _f(x), _f(w)
    out = np.empty_like(x)
    _check(lib().s2o_rms_norm_heads(_p(x), _p(w), x.size, head_dim, eps, _p(out)))
    return out


def linear(x, w, in_dim, out_dim):
    x, w = _f(x), _f(w)
    if x.size != in_dim:
        raise OracleError(f"linear input length mismatch: expected {in_dim}, got {x.size}")
    if w.size != in_dim * out_dim:
        raise OracleError(f"linear weight length mismatch: expected {in_dim * out_dim}, "
                          f"got {w.size}")
    out = np.empty(out_dim, dtype=np.float32)
    _check(lib().s2o_linear(_p(x), _p(w), in_dim, out_dim, _p(out)))
    return out


def matvec_f16(x, w_bits, in_dim, out_dim):
    x = _f(x)
    w = np.ascontiguousarray(np.asarray(w_bits, dtype=np.uint16))
    if x.size != in_dim:
        raise OracleError(f"matvec_f16_streaming input length mismatch: expected {in_dim}, "
                          f"got {x.size}")
    if w.size != in_dim * out_dim:
        raise OracleError("matvec_f16_streaming weight byte length mismatch")
    out = np.empty(out_dim, dtype=np.float32)
    _check(lib().s2o_matvec_f16(_p(x), _p(w, ctypes.c_uint16), in_dim, out_dim, _p(out)))
    return out


def rope_normal(values, head_dim, position, base):
    v = _f(values).copy()
    _check(lib().s2o_rope_normal(_p(v), v.size, head_dim, position, base))
    return v


def gqa_decode_attention(q, k, v, H, Hkv, hd, T, scale):
    q, k, v = _f(q), _f(k), _f(v)
    out = np.empty(H * hd, dtype=np.float32)
    _check(lib().s2o_gqa_decode_attention(_p(q), _p(k), _p(v), H, Hkv, hd, T, scale, _p(out)))
    return out


def swiglu_slow(g, u):
    g, u = _f(g), _f(u)
    out = np.empty_like(g)
    _check(lib().s2o_swiglu_slow(_p(g), _p(u), g.size, _p(out)))
    return out


def swiglu_fast(g, u):
    g, u = _f(g), _f(u)
    out = np.empty_like(g)
    _check(lib().s2o_swiglu_fast(_p(g), _p(u), g.size, _p(out)))
    return out


class SeededRng:
    def __init__(self, seed: int):
        self.state = ctypes.c_uint64(seed)

    def next_unit(self) -> float:
        return lib().s2o_rng_next_unit(ctypes.byref(self.state))


def build_semantic_bias(vocab, sem_begin, sem_end, im_end_id=None):
    out = np.empty(vocab, dtype=np.float32)
    _check(lib().s2o_build_semantic_bias(vocab, sem_begin, sem_end,
                                         -1 if im_end_id is None else im_end_id, _p(out)))
    return out


def apply_semantic_bias(logits, bias, block_im_end, im_end_id=None):
    lg, b = _f(logits).copy(), _f(bias)
    if lg.size != b.size:
        raise OracleError(f"semantic bias length mismatch: logits={lg.size} bias={b.size}")
    _check(lib().s2o_apply_semantic_bias(_p(lg), _p(b), lg.size, int(block_im_end),
                                         -1 if im_end_id is None else im_end_id))
    return lg


def semantic_mask_logits(logits, sem_begin, sem_end, im_end_id, block_im_end):
    lg = _f(logits).copy()
    _check(lib().s2o_semantic_mask_logits(_p(lg), lg.size, sem_begin, sem_end,
                                          -1 if im_end_id is None else im_end_id,
                                          int(block_im_end)))
    return lg


def sample_token(logits, temperature, top_p, top_k, always_include_id, rng: SeededRng) -> int:
    lg = _f(logits)
    out = ctypes.c_uint32()
    _check(lib().s2o_sample_token(_p(lg), lg.size, temperature, top_p, top_k,
                                  -1 if always_include_id is None else always_include_id,
                                  ctypes.byref(rng.state), ctypes.byref(out)))
    return int(out.value)


# ---- KV cache + toy layer (attention.rs, slow_ar.rs skeleton) --------------

class KvCache:
    def __init__(self, head_dim, head_count_kv, max_seq, layers):
        self.hd, self.hkv = head_dim, head_count_kv
        self._p = lib().s2o_kv_new(head_dim, head_count_kv, max_seq, layers)
        if not self._p:
            raise OracleError(lib().s2o_last_error().decode())

    def __del__(self):
        if getattr(self, "_p", None):
            lib().s2o_kv_free(self._p)
            self._p = None

    def write_token(self, layer, token, key, value):
        _check(lib().s2o_kv_write_token(self._p, layer, token, _p(_f(key)), _p(_f(value))))

    def read_token(self, layer, token):
        k = np.empty(self.hd * self.hkv, dtype=np.float32)
        v = np.empty_like(k)
        _check(lib().s2o_kv_read_token(self._p, layer, token, _p(k), _p(v)))
        return k, v

    def decode_attention(self, layer, token_count, query, head_count, scale):
        q = _f(query)
        out = np.empty(head_count * self.hd, dtype=np.float32)
        _check(lib().s2o_kv_decode_attention(self._p, layer, token_count, _p(q), head_count,
                                             scale, _p(out)))
        return out


def layer_forward(shape: dict, weights: dict, hidden_tokens, kv: KvCache, layer=0, start=0,
                  decode_loop=False, trace=True):
    """SlowArLayerSkeleton over toy f32 weights; returns (hidden, trace dict)."""
    sh = LayerShape(**shape)
    ws = {k: _f(v) for k, v in weights.items()}
    lw = LayerWeights(**{n: _p(ws[n]) for n in _W_NAMES}, **{"n_" + n: ws[n].size for n in _W_NAMES})
    x = _f(hidden_tokens)
    n = x.size // shape["hidden_size"]
    d, F = shape["hidden_size"], shape["feed_forward_size"]
    qs, kvs = shape["head_count"] * shape["head_dim"], shape["head_count_kv"] * shape["head_dim"]
    widths = dict(normalized=d, query=qs, key=kvs, value=kvs, attention=qs, projected=d,
                  attn_hidden=d, ffn_normalized=d, gate=F, up=F, activated=F, ffn_projected=d,
                  hidden=d)
    bufs = {k: np.zeros(n * w, dtype=np.float32) for k, w in widths.items()}
    tr = LayerTrace(**{k: _p(b) for k, b in bufs.items()}) if trace else None
    out = np.empty_like(x)
    _check(lib().s2o_layer_forward(ctypes.byref(sh), ctypes.byref(lw), _p(x), n, kv._p, layer,
                                   start, int(decode_loop), ctypes.byref(tr) if tr else None,
                                   _p(out)))
    return out, {k: b.reshape(n, -1) for k, b in bufs.items()}


# ---- model ----------------------------------------------------------------

class OracleModel:
    """SlowArState + FastArWeights over a GGUF file on the CPU.
    mode 0: resident (fast); mode 1: reference-faithful timing."""

    def __init__(self, path, max_seq_len=4096, mode=0):
        self._p = lib().s2o_open(str(path).encode(), max_seq_len, mode)
        if not self._p:
            raise OracleError(lib().s2o_last_error().decode(errors="replace"))
        self.spec = GraphSpec()
        _check(lib().s2o_graph_spec(self._p, ctypes.byref(self.spec)))

    def close(self):
        if getattr(self, "_p", None):
            lib().s2o_close(self._p)
            self._p = None

    def __del__(self):
        self.close()

    def reset(self):
        lib().s2o_reset(self._p)

    def n_past(self) -> int:
        return int(lib().s2o_n_past(self._p))

    def eval(self, flat, logits=True, allowed_only=False, im_end_id=None):
        toks = np.ascontiguousarray(np.asarray(flat, dtype=np.int32))
        hidden = np.empty(self.spec.slow_embedding_length, dtype=np.float32)
        lg = np.empty(self.spec.vocab_size, dtype=np.float32) if logits else None
        _check(lib().s2o_eval(self._p, _p(toks, ctypes.c_int32), toks.size, _p(hidden), _p(lg),
                              int(allowed_only), -1 if im_end_id is None else im_end_id))
        return hidden, lg

    def fast_prefix_logits(self, slow_hidden, prefix):
        h = _f(slow_hidden)
        pre = np.ascontiguousarray(np.asarray(prefix, dtype=np.uint32))
        out = np.empty(self.spec.codebook_size, dtype=np.float32)
        _check(lib().s2o_fast_prefix_logits(self._p, _p(h), _p(pre, ctypes.c_uint32), pre.size,
                                            _p(out)))
        return out

    def generate_codebooks(self, slow_hidden, semantic_code, temperature, top_p, top_k,
                           rng: SeededRng):
        h = _f(slow_hidden)
        out = np.empty(self.spec.num_codebooks, dtype=np.uint32)
        _check(lib().s2o_generate_codebooks(self._p, _p(h), semantic_code, temperature, top_p,
                                            top_k, ctypes.byref(rng.state),
                                            _p(out, ctypes.c_uint32)))
        return [int(x) for x in out]

    def generate_codes(self, prompt: np.ndarray, params: dict, rng: SeededRng):
        """prompt: (K+1) x cols uint32.  Returns (codes[K, n_frames], mains)."""
        p = np.ascontiguousarray(np.asarray(prompt, dtype=np.uint32))
        rows, cols = p.shape
        k = max(self.spec.num_codebooks, 1)
        mx = params["max_new_tokens"]
        codes = np.zeros(k * max(mx, 1), dtype=np.int32)
        mains = np.zeros(mx + 1, dtype=np.uint32)
        gp = GenParams(**params)
        nf = ctypes.c_uint32()
        _check(lib().s2o_generate_codes(self._p, _p(p, ctypes.c_uint32), rows, cols,
                                        ctypes.byref(gp), ctypes.byref(rng.state),
                                        _p(codes, ctypes.c_int32), ctypes.byref(nf),
                                        _p(mains, ctypes.c_uint32)))
        n = int(nf.value)
        return codes[: k * n].reshape(k, n), mains[: n + 1]


def set_threads(n: int) -> int:
    return lib().s2o_set_threads(n)


def get_threads() -> int:
    return lib().s2o_get_threads()


# ---- GGUF ------------------------------------------------------------------

class Gguf:
    def __init__(self, path):
        self._p = lib().s2o_gguf_open(str(path).encode())
        if not self._p:
            raise OracleError(lib().s2o_last_error().decode(errors="replace"))

    def __del__(self):
        if getattr(self, "_p", None):
            lib().s2o_gguf_close(self._p)
            self._p = None

    @property
    def version(self) -> int:
        return lib().s2o_gguf_version(self._p)

    @property
    def data_start(self) -> int:
        return lib().s2o_gguf_data_start(self._p)

    def tensors(self):
        out = []
        for i in range(lib().s2o_gguf_tensor_count(self._p)):
            name = ctypes.c_char_p()
            rank = ctypes.c_int32()
            dims = (ctypes.c_uint64 * 4)()
            t = ctypes.c_uint32()
            rel = ctypes.c_uint64()
            nb = ctypes.c_uint64()
            _check(lib().s2o_gguf_tensor_info(self._p, i, ctypes.byref(name), ctypes.byref(rank),
                                              dims, ctypes.byref(t), ctypes.byref(rel),
                                              ctypes.byref(nb)))
            out.append(dict(name=name.value.decode(), dims=list(dims[: rank.value]),
                            type=t.value, rel_offset=rel.value, bytes=nb.value))
        return out

    def tensor_bytes(self, name) -> bytes:
        n = ctypes.c_uint64()
        p = lib().s2o_gguf_tensor_data(self._p, name.encode(), ctypes.byref(n))
        if not p:
            raise OracleError(lib().s2o_last_error().decode())
        return ctypes.string_at(p, n.value)

    def metadata(self, key) -> str:
        buf = ctypes.create_string_buffer(4096)
        _check(lib().s2o_gguf_metadata(self._p, key.encode(), buf, len(buf)))
        return buf.value.decode()


def dequant(ggml_type: int, raw: bytes, n: int) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    buf = ctypes.create_string_buffer(raw, len(raw))
    _check(lib().s2o_dequant_row(ggml_type, buf, n, _p(out)))
    return out
