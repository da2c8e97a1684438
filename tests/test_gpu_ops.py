"""Op-level parity of the sm_100a kernels against the CPU oracle, through the
C ABI (the MatmulBackend seam, backend.rs:5-121, and sample_token,
sampling.rs:121-200)."""
import math

import numpy as np
import pytest

from oracle import oracle as o

pytestmark = pytest.mark.gpu

F32 = np.float32


@pytest.fixture(scope="module")
def backend():
    from fish_s2pro_b200 import CudaMatmulBackend
    return CudaMatmulBackend()


def rel_err(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


@pytest.mark.parametrize("k,n", [(512, 768), (2560, 6144), (4096, 2560), (9728, 64), (8, 3)])
def test_linear_f16_matches_oracle(backend, k, n):
    rng = np.random.default_rng(k + n)
    x = rng.standard_normal(k).astype(F32)
    w = (rng.standard_normal(k * n) * 0.02).astype(np.float16).view(np.uint16)
    got = backend.linear_f16(x, w, k, n)
    want = o.matvec_f16(x, w, k, n)
    assert rel_err(got, want) < 1e-5


def test_linear_rejects_bad_shapes(backend):
    from fish_s2pro_b200 import S2dError
    with pytest.raises(S2dError, match="weight length mismatch"):
        backend.linear_f16(np.ones(8, F32), np.zeros(7, np.uint16), 8, 1)


@pytest.mark.parametrize("n,hd", [(2560, 2560), (4096, 128), (1024, 128), (512, 64)])
def test_rms_norm_heads_matches_oracle(backend, n, hd):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(F32) * 3
    w = rng.uniform(0.5, 1.5, hd).astype(F32)
    got = backend.rms_norm_heads(x, w, hd, 1e-6)
    want = o.rms_norm_heads(x, w, hd, 1e-6)
    assert np.max(np.abs(got - want)) <= 4e-6 * np.max(np.abs(want))


@pytest.mark.parametrize("heads,hd,pos,base", [(32, 128, 0, 1e6), (32, 128, 511, 1e6), (8, 128, 8191, 1e6),
                                               (4, 64, 10, 1e4), (2, 256, 30000, 1e6)])
def test_rope_normal_matches_oracle(backend, heads, hd, pos, base):
    """apply_rope_normal (attention.rs:172-206) on the per-op/rows RoPE: the
    rotation's sin and cos come from CUDA's sincosf where the reference calls
    f32 sin_cos, so the tolerance is a few f32 ulps of the largest value."""
    rng = np.random.default_rng(pos + heads)
    x = rng.standard_normal(heads * hd).astype(F32)
    got = backend.apply_rope_normal(x, hd, pos, base)
    want = o.rope_normal(x, hd, pos, base)
    assert rel_err(got, want) < 2e-6
    # the rotation keeps every pair's length
    a, b = got.reshape(-1, 2).astype(np.float64), x.reshape(-1, 2).astype(np.float64)
    np.testing.assert_allclose(np.hypot(a[:, 0], a[:, 1]), np.hypot(b[:, 0], b[:, 1]), rtol=1e-5)


def test_rope_normal_kat(backend):  # attention.rs:336-343 at head_dim 64
    x = np.zeros(64, F32)
    x[0], x[3] = 1.0, 1.0
    got = backend.apply_rope_normal(x, 64, 1, 10_000.0)
    want = o.rope_normal(x, 64, 1, 10_000.0)
    np.testing.assert_allclose(got, want, atol=1e-6)
    assert abs(got[0] - math.cos(1.0)) < 1e-6 and abs(got[1] - math.sin(1.0)) < 1e-6


@pytest.mark.parametrize("H,Hkv,hd,T", [(4, 2, 64, 1), (32, 8, 128, 7), (32, 8, 128, 700),
                                       (8, 2, 64, 129), (16, 16, 128, 33)])
def test_gqa_attention_matches_oracle(backend, H, Hkv, hd, T):
    rng = np.random.default_rng(T * 7 + H)
    q = rng.standard_normal(H * hd).astype(F32)
    k = rng.standard_normal(T * Hkv * hd).astype(F32)
    v = rng.standard_normal(T * Hkv * hd).astype(F32)
    scale = F32(1.0) / np.sqrt(F32(hd))
    got = backend.gqa_decode_attention(q, k, v, H, Hkv, hd, T, float(scale))
    want = o.gqa_decode_attention(q, k, v, H, Hkv, hd, T, float(scale))
    assert rel_err(got, want) < 2e-5


def test_gqa_attention_kat(backend):  # attention.rs:362-406 with head_dim 64
    hd = 64
    q = np.zeros(4 * hd, F32)
    q[0] = q[hd + 1] = q[2 * hd] = q[3 * hd + 1] = 1
    k = np.zeros(2 * 2 * hd, F32)
    k[0] = k[hd + 1] = k[2 * hd + 1] = k[3 * hd] = 1
    v = np.zeros(2 * 2 * hd, F32)
    v[0], v[hd + 1], v[2 * hd], v[3 * hd + 1] = 10, 10, 20, 20
    out = backend.gqa_decode_attention(q, k, v, 4, 2, hd, 2, 1.0).reshape(4, hd)
    p_hi = math.exp(1) / (math.exp(1) + 1.0)
    p_lo = 1 - p_hi
    assert out[0, 0] == pytest.approx(10 * p_hi + 20 * p_lo, abs=1e-5)
    assert out[1, 0] == pytest.approx(10 * p_lo + 20 * p_hi, abs=1e-5)
    assert out[2, 1] == pytest.approx(10 * p_lo + 20 * p_hi, abs=1e-5)
    assert out[3, 1] == pytest.approx(10 * p_hi + 20 * p_lo, abs=1e-5)


# ---- device sampler: exact token and RNG stream ------------------------------

SAMPLER_CASES = [
    # temperature, top_p, top_k
    (0.0, 1.0, 0),
    (0.0, 1.0, 1),
    (0.0, 0.5, 5),
    (0.7, 0.7, 30),
    (0.8, 0.9, 30),
    (1.0, 1.0, 0),
    (1.3, 0.95, 200),
    (0.5, 0.3, 3),
    (0.9, 0.99, 256),  # the largest top-k of the radix-select path
    (0.9, 1.0, 257),   # the smallest top-k of the full sort
]


def _logit_vectors(rng, n):
    a = rng.standard_normal(n).astype(F32) * 2
    b = a.copy()
    b[rng.integers(0, n, max(1, n // 10))] = -np.inf          # masked entries
    c = np.round(a * 2) / 2                                    # many exact ties
    d = np.full(n, -np.inf, F32)                               # all masked
    e = a.copy()
    e[3 % n] = e.max() + 1e-7                                  # near tie within 1e-6
    return [a, b, c.astype(F32), d, e]


@pytest.fixture(scope="module")
def tiny_state(tiny_gguf):
    from fish_s2pro_b200 import SlowArState
    st = SlowArState.open(tiny_gguf, max_seq_len=256)
    yield st
    st.close()


@pytest.mark.parametrize("n", [1, 5, 100, 1024, 4097, 8192])
def test_sampler_matches_oracle_exactly(tiny_state, n):
    from fish_s2pro_b200 import SamplerParams, SeededRng, sample_token
    rng = np.random.default_rng(n)
    for lg in _logit_vectors(rng, n):
        for t, p, k in SAMPLER_CASES:
            for force in (None, int(rng.integers(0, n))):
                seed = int(rng.integers(0, 2**63))
                g_rng, o_rng = SeededRng(seed), o.SeededRng(seed)
                got = sample_token(tiny_state, lg, SamplerParams(t, p, k), force, g_rng)
                want = o.sample_token(lg, t, p, k, force, o_rng)
                assert got == want, (n, t, p, k, force)
                assert g_rng.state == o_rng.state.value
