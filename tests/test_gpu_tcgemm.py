"""The rows path's tcgen05 GEMM (s2d_op_rows_linear_f16, impl 0) against a
plain float64 reference of the same op, and against the cuBLAS + combine
path (impl 1).

y[t][n] = epi(sum_k x[t][k] * w[n][k]) with f16 weights and f32 rows; the
rows enter the tensor cores as f16 hi + lo halves (about 22 bits), so the
GEMM matches the float reference to ~1e-6 relative; the bound below
(2e-5 x max|y|) is far under what any layout or descriptor error gives.
Shapes cover token tiles of 64 / 128 (several per call), split-K clusters (few row
tiles, long K), row and token tails, and every epilogue.
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


def run(st, x, w, w2=None, resid=None, epi=0, impl=0):
    import ctypes

    from fish_s2pro_b200 import lib
    from fish_s2pro_b200.s2d import _P
    T, K = x.shape
    N = w.shape[0]
    y = np.zeros((T, N), dtype=np.float32)
    f32, u16 = _P(ctypes.c_float), _P(ctypes.c_uint16)
    p = lambda a, t: a.ctypes.data_as(t) if a is not None else None  # noqa: E731
    rc = lib().s2d_op_rows_linear_f16(st.handle, p(x, f32), T, K, p(w, u16), p(w2, u16), N,
                                      p(resid, f32), epi, impl, p(y, f32))
    assert rc == 0, lib().s2d_last_error(st.handle)
    return y


def reference(x, wf, w2f, resid, epi):
    v = x.astype(np.float64) @ wf.T
    if epi == 0:
        return v
    if epi == 1:
        return resid.astype(np.float64) + v
    u = x.astype(np.float64) @ w2f.T
    return v / (1.0 + np.exp(-v)) * u


SHAPES = [  # T, K, N
    (1, 64, 128), (5, 512, 200), (64, 512, 1536), (64, 2560, 2560), (64, 4096, 2560),
    (100, 1536, 512), (128, 512, 768), (128, 2560, 640), (300, 512, 384), (512, 2560, 256),
    (64, 2560, 6144), (64, 2560, 9728),  # the batched step's WQKV and w1 / w3 shapes
]


@pytest.mark.parametrize("T,K,N", SHAPES)
@pytest.mark.parametrize("epi", [0, 1, 2, 3])
def test_tcgemm_matches_float_reference(st, T, K, N, epi):
    rng = np.random.default_rng(T * 131 + K * 7 + N + epi)
    x = rng.standard_normal((T, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float16)
    w2 = (rng.standard_normal((N, K)) * 0.05).astype(np.float16) if epi >= 2 else None
    resid = rng.standard_normal((T, N)).astype(np.float32) if epi == 1 else None
    want = reference(x, w.astype(np.float64), None if w2 is None else w2.astype(np.float64), resid, epi)
    got = run(st, x, w.view(np.uint16), None if w2 is None else w2.view(np.uint16), resid, epi, impl=0)
    err = np.max(np.abs(got - want)) / np.max(np.abs(want))
    assert err < TOL, (T, K, N, epi, err)
    if epi in (0, 2):
        lib_path = run(st, x, w.view(np.uint16), None if w2 is None else w2.view(np.uint16), resid, epi, impl=1)
        assert np.max(np.abs(got - lib_path)) / np.max(np.abs(want)) < TOL


def test_tcgemm_rejects_k_not_multiple_of_64(st):
    from fish_s2pro_b200 import lib
    import ctypes
    from fish_s2pro_b200.s2d import _P
    x = np.ones((4, 72), dtype=np.float32)
    w = np.ones((128, 72), dtype=np.float16).view(np.uint16)
    y = np.zeros((4, 128), dtype=np.float32)
    rc = lib().s2d_op_rows_linear_f16(st.handle, x.ctypes.data_as(_P(ctypes.c_float)), 4, 72,
                                      w.ctypes.data_as(_P(ctypes.c_uint16)), None, 128, None, 0, 0,
                                      y.ctypes.data_as(_P(ctypes.c_float)))
    assert rc != 0
