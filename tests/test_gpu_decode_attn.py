"""The batched Slow-AR step's attention (s2d_op_batch_attention) against a
plain float64 restatement of gqa_decode_attention + softmax_in_place
(attention.rs:208-309), once per sequence: impl 0 is the tensor-core kernel,
impl 1 the CUDA-core rows kernel.

K / V are f16 (the cache type); the tensor-core kernel feeds q and the
softmax weights to the MMAs as f16 hi + lo pairs (about 22 bits) with f32
accumulation, so both kernels match the float64 result to ~1e-6 of
max|out|; the bound below (2e-5) is far under what a fragment-layout,
masking or merge error gives.  Cases cover head dims 64 / 128, GQA groups of
1, 2, 4 and 8 heads, context lengths from 1 to past 4,000 positions (partial
last chunks, more warps and splits than chunks), explicit split counts, and
finished sequences.

The prompt-chunk attention (s2d_op_prefill_attention, the attention of
forward_prefill_sequence, slow_ar.rs:579-593) is checked the same way for its
three kernels: impl 0 the mma.sync tensor-core kernel, 1 the CUDA-core
kernels, 2 the tcgen05 kernel (TMEM accumulators, head dim 128), which also
feeds q and the softmax weights as f16 hi + lo pairs.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-5


@pytest.fixture(scope="module")
def st(tiny_gguf):
    from fish_s2pro_b200 import SlowArState
    s = SlowArState.open(tiny_gguf, max_seq_len=64)
    yield s
    s.close()


def run(st, q, k, v, n_past, done=None, splits=0, impl=0):
    import ctypes

    from fish_s2pro_b200 import lib
    from fish_s2pro_b200.s2d import _P
    B, H, hd = q.shape
    Hkv, max_seq = k.shape[1], k.shape[2]
    out = np.zeros_like(q)
    i32 = _P(ctypes.c_int32)
    npast = np.ascontiguousarray(n_past, dtype=np.int32)
    dn = None if done is None else np.ascontiguousarray(done, dtype=np.int32)
    rc = lib().s2d_op_batch_attention(
        st.handle, q.ctypes.data_as(_P(ctypes.c_float)), k.view(np.uint16).ctypes.data_as(_P(ctypes.c_uint16)),
        v.view(np.uint16).ctypes.data_as(_P(ctypes.c_uint16)), B, H, Hkv, hd, max_seq, npast.ctypes.data_as(i32),
        None if dn is None else dn.ctypes.data_as(i32), splits, impl, out.ctypes.data_as(_P(ctypes.c_float)))
    assert rc == 0, lib().s2d_last_error(st.handle)
    return out


def reference(q, k, v, n_past, done=None):
    B, H, hd = q.shape
    rep = H // k.shape[1]
    out = np.zeros((B, H, hd))
    for b in range(B):
        if done is not None and done[b]:
            continue
        n = int(n_past[b]) + 1
        for h in range(H):
            kk = k[b, h // rep, :n].astype(np.float64)
            s = kk @ q[b, h].astype(np.float64) / np.sqrt(hd)
            p = np.exp(s - s.max())
            out[b, h] = (p / p.sum()) @ v[b, h // rep, :n].astype(np.float64)
    return out


def case(B, H, Hkv, hd, max_seq, seed):
    rng = np.random.default_rng(seed)
    q = (rng.standard_normal((B, H, hd)) * 2.0).astype(np.float32)
    k = rng.standard_normal((B, Hkv, max_seq, hd)).astype(np.float16)
    v = rng.standard_normal((B, Hkv, max_seq, hd)).astype(np.float16)
    return q, k, v


CASES = [  # B, H, Hkv, hd, max_seq, positions
    (2, 8, 2, 64, 64, (0, 63)),
    (3, 32, 8, 128, 160, (1, 31, 159)),
    (4, 32, 8, 128, 1100, (1000, 33, 64, 1099)),
    (2, 8, 8, 128, 300, (299, 17)),
    (2, 16, 2, 64, 4200, (4199, 2500)),
    (3, 8, 1, 128, 120, (119, 0, 64)),  # one kv head for 8 query heads
]


@pytest.mark.parametrize("B,H,Hkv,hd,max_seq,pos", CASES)
@pytest.mark.parametrize("impl", [0, 1])
def test_batch_attention_matches_float_reference(st, B, H, Hkv, hd, max_seq, pos, impl):
    q, k, v = case(B, H, Hkv, hd, max_seq, B * 7 + H + hd + max_seq)
    want = reference(q, k, v, pos)
    got = run(st, q, k, v, pos, impl=impl)
    err = np.max(np.abs(got - want)) / np.max(np.abs(want))
    assert err < TOL, err


@pytest.mark.parametrize("splits", [1, 2, 7, 40])
def test_batch_attention_split_counts(st, splits):
    q, k, v = case(3, 32, 8, 128, 700, splits)
    pos = (699, 5, 300)
    want = reference(q, k, v, pos)
    got = run(st, q, k, v, pos, splits=splits, impl=0)
    assert np.max(np.abs(got - want)) / np.max(np.abs(want)) < TOL


def test_batch_attention_skips_finished_sequences(st):
    q, k, v = case(3, 32, 8, 128, 200, 9)
    pos, done = (150, 199, 60), (0, 1, 0)
    got = run(st, q, k, v, pos, done=done, impl=0)
    assert not np.any(got[1])
    want = reference(q, k, v, pos, done)
    assert np.max(np.abs(got - want)) / np.max(np.abs(want)) < TOL


def test_batch_attention_large_scores(st):
    """Queries of large magnitude (scores spanning hundreds of units): the
    power-of-two pre-scaling keeps the f16 halves in range."""
    q, k, v = case(2, 32, 8, 128, 400, 3)
    q *= 300.0
    pos = (399, 128)
    want = reference(q, k, v, pos)
    got = run(st, q, k, v, pos, impl=0)
    assert np.max(np.abs(got - want)) / np.max(np.abs(want)) < TOL


def test_batch_attention_rejects_bad_arguments(st):
    q, k, v = case(2, 8, 2, 64, 32, 0)
    from fish_s2pro_b200 import lib
    import ctypes
    from fish_s2pro_b200.s2d import _P
    npast = np.array([40, 0], dtype=np.int32)  # past max_seq
    out = np.zeros_like(q)
    rc = lib().s2d_op_batch_attention(
        st.handle, q.ctypes.data_as(_P(ctypes.c_float)), k.view(np.uint16).ctypes.data_as(_P(ctypes.c_uint16)),
        v.view(np.uint16).ctypes.data_as(_P(ctypes.c_uint16)), 2, 8, 2, 64, 32,
        npast.ctypes.data_as(_P(ctypes.c_int32)), None, 0, 0, out.ctypes.data_as(_P(ctypes.c_float)))
    assert rc != 0


@pytest.mark.parametrize("env", [
    {"S2D_DECODE_CHUNK": "32"},
    {"S2D_DECODE_CHUNK": "32", "S2D_DECODE_STAGES": "3"},
    {"S2D_DECODE_WARPS": "2", "S2D_DECODE_STAGES": "3"},
])
def test_batch_attention_kernel_variants(tiny_gguf, monkeypatch, env):
    """The chunk / ring / warp variants (selected when a state opens)."""
    from fish_s2pro_b200 import SlowArState
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    s = SlowArState.open(tiny_gguf, max_seq_len=64)
    try:
        for B, H, Hkv, hd, max_seq, pos in (CASES[1], CASES[2], CASES[4]):
            q, k, v = case(B, H, Hkv, hd, max_seq, 5)
            want = reference(q, k, v, pos)
            got = run(s, q, k, v, pos, impl=0)
            assert np.max(np.abs(got - want)) / np.max(np.abs(want)) < TOL
    finally:
        s.close()


# ---- prompt-chunk (prefill) attention ---------------------------------------

def run_prefill(st, q, k, v, pos0, impl):
    import ctypes

    from fish_s2pro_b200 import lib
    from fish_s2pro_b200.s2d import _P
    T, H, hd = q.shape
    Hkv, max_seq = k.shape[0], k.shape[1]
    out = np.zeros_like(q)
    rc = lib().s2d_op_prefill_attention(
        st.handle, q.ctypes.data_as(_P(ctypes.c_float)), k.view(np.uint16).ctypes.data_as(_P(ctypes.c_uint16)),
        v.view(np.uint16).ctypes.data_as(_P(ctypes.c_uint16)), T, H, Hkv, hd, max_seq, pos0, impl,
        out.ctypes.data_as(_P(ctypes.c_float)))
    assert rc == 0, lib().s2d_last_error(st.handle)
    return out


def reference_prefill(q, k, v, pos0):
    T, H, hd = q.shape
    rep = H // k.shape[0]
    out = np.zeros((T, H, hd))
    for m in range(T):
        n = pos0 + m + 1
        for h in range(H):
            s = k[h // rep, :n].astype(np.float64) @ q[m, h].astype(np.float64) / np.sqrt(hd)
            p = np.exp(s - s.max())
            out[m, h] = (p / p.sum()) @ v[h // rep, :n].astype(np.float64)
    return out


PREFILL_CASES = [  # T, H, Hkv, hd, max_seq, pos0
    (16, 8, 2, 64, 64, 0),
    (40, 32, 8, 128, 96, 0),
    (37, 32, 8, 128, 200, 100),   # a later chunk, ragged tile
    (64, 16, 2, 64, 700, 600),
    (33, 8, 8, 128, 80, 7),       # one head per group (8 tokens per warp)
    (48, 16, 8, 128, 90, 20),     # two heads per group
    (20, 8, 1, 64, 50, 30),       # eight heads per group (one token per warp)
    (256, 32, 8, 128, 1400, 1100),  # a long context: 22 position tiles of 64, 8 query tiles
    (130, 32, 4, 128, 300, 150),  # eight heads per group: 16 tokens per tcgen05 tile, ragged
    (16, 32, 32, 128, 40, 0),     # one head per group: 128 tokens per tcgen05 tile, one partial tile
]


# impl 0: mma.sync tensor-core kernel, 1: CUDA cores, 2: tcgen05 (head dim 128 only)
@pytest.mark.parametrize("T,H,Hkv,hd,max_seq,pos0", PREFILL_CASES)
@pytest.mark.parametrize("impl", [0, 1, 2])
def test_prefill_attention_matches_float_reference(st, T, H, Hkv, hd, max_seq, pos0, impl):
    if impl == 2 and hd != 128:
        pytest.skip("the tcgen05 kernel takes head dim 128")
    rng = np.random.default_rng(T * 3 + H + hd + pos0)
    q = (rng.standard_normal((T, H, hd)) * 2.0).astype(np.float32)
    k = rng.standard_normal((Hkv, max_seq, hd)).astype(np.float16)
    v = rng.standard_normal((Hkv, max_seq, hd)).astype(np.float16)
    want = reference_prefill(q, k, v, pos0)
    got = run_prefill(st, q, k, v, pos0, impl)
    assert np.max(np.abs(got - want)) / np.max(np.abs(want)) < TOL


@pytest.mark.parametrize("T,H,Hkv,max_seq,pos0", [(64, 32, 8, 200, 100), (130, 32, 4, 300, 150)])
@pytest.mark.parametrize("impl", [0, 1, 2])
def test_prefill_attention_rising_scores(st, T, H, Hkv, max_seq, pos0, impl):
    """Key rows whose norm grows with the position: each row's max score
    climbs by several base-2 units per 64-position tile (scores reach ~75),
    so the tcgen05 kernel's online softmax moves its reference max and
    rescales the accumulator in TMEM one to four times per row of the last
    token; a key aligned with the last token's q sits mid-chunk on top."""
    hd = 128
    rng = np.random.default_rng(T + pos0)
    q = (rng.standard_normal((T, H, hd)) * 2.0).astype(np.float32)
    grow = (0.3 + 2.5 * np.arange(max_seq) / 64.0)[None, :, None]
    k = (rng.standard_normal((Hkv, max_seq, hd)) * grow).astype(np.float16)
    v = rng.standard_normal((Hkv, max_seq, hd)).astype(np.float16)
    spike = pos0 + T // 2
    k[:, spike] = (np.sign(q[T - 1, ::H // Hkv]) * 1.5).astype(np.float16)
    want = reference_prefill(q, k, v, pos0)
    got = run_prefill(st, q, k, v, pos0, impl)
    assert np.max(np.abs(got - want)) / np.max(np.abs(want)) < TOL
