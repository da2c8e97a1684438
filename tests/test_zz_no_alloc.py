"""The allocation-free attention entry point, for callers that cannot call
cudaMalloc (a real-time audio thread must not block in the CUDA allocator; a
host with a fixed device-memory budget owns every allocation itself).

It is called through the C ABI with caller-owned device buffers, twice in a
row (its fixed scratch keeps the previous call's contents), and must agree
with the CPU oracle's gqa_decode_attention (attention.rs:208-247) and with the
allocating s2d_op_gqa_decode_attention.  This file sorts last so that a run
stopping at the first failure has run every other test first.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-5  # the attention tolerance of tests/test_gpu_ops.py


def rel_err(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def _call(lib, q, k, v, H, Hkv, hd, T, scale, out, stream):
    err = ctypes.create_string_buffer(512)
    rc = lib.s2d_op_gqa_decode_attention_noalloc(q, k, v, H, Hkv, hd, T, scale, out, stream, err,
                                                 len(err))
    return rc, err.value.decode()


@pytest.mark.parametrize("H,Hkv,hd,T", [(32, 8, 128, 700), (8, 2, 64, 33), (4, 2, 64, 1)])
def test_noalloc_attention_matches_oracle(H, Hkv, hd, T):
    import torch

    from fish_s2pro_b200 import CudaMatmulBackend, s2d
    from oracle import oracle as o
    lib = s2d.lib()
    rng = np.random.default_rng(H * 1000 + T)
    q = rng.standard_normal(H * hd).astype(np.float32)
    k = rng.standard_normal(T * Hkv * hd).astype(np.float32)
    v = rng.standard_normal(T * Hkv * hd).astype(np.float32)
    scale = float(np.float32(1.0) / np.sqrt(np.float32(hd)))
    want = o.gqa_decode_attention(q, k, v, H, Hkv, hd, T, scale)
    alloc = CudaMatmulBackend().gqa_decode_attention(q, k, v, H, Hkv, hd, T, scale)

    dev = torch.device("cuda", 0)
    dq = torch.from_numpy(q).to(dev)
    # the entry point takes keys/values head-major: [head_count_kv][token_count][head_dim]
    dk = torch.from_numpy(k.reshape(T, Hkv, hd).transpose(1, 0, 2).copy()).to(dev)
    dv = torch.from_numpy(v.reshape(T, Hkv, hd).transpose(1, 0, 2).copy()).to(dev)
    dout = torch.empty(H * hd, dtype=torch.float32, device=dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    for _ in range(2):
        dout.fill_(float("nan"))
        rc, msg = _call(lib, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), H, Hkv, hd, T, scale,
                        dout.data_ptr(), stream)
        assert rc == 0, msg
        got = dout.cpu().numpy()
        assert rel_err(got, want) < TOL
        assert rel_err(got, alloc) < TOL


def test_noalloc_attention_rejects_sizes_beyond_its_scratch():
    import torch

    from fish_s2pro_b200 import s2d
    lib = s2d.lib()
    H, Hkv, hd, T = 64, 4, 256, 1024  # 64 * 16 * 258 floats > 131072
    dev = torch.device("cuda", 0)
    buf = torch.zeros(H * hd, dtype=torch.float32, device=dev)
    kv = torch.zeros(Hkv * T * hd, dtype=torch.float32, device=dev)
    rc, msg = _call(lib, buf.data_ptr(), kv.data_ptr(), kv.data_ptr(), H, Hkv, hd, T, 0.0625,
                    buf.data_ptr(), None)
    assert rc == -1
    assert "limit" in msg


def test_noalloc_attention_rejects_misaligned_keys():
    """A view that starts one float into its buffer cannot be read as float4:
    the call returns S2D_EINVAL before any device work."""
    import torch

    from fish_s2pro_b200 import s2d
    lib = s2d.lib()
    H, Hkv, hd, T = 8, 2, 128, 16
    dev = torch.device("cuda", 0)
    q = torch.zeros(H * hd, dtype=torch.float32, device=dev)
    kv = torch.zeros(Hkv * T * hd + 1, dtype=torch.float32, device=dev)
    out = torch.zeros(H * hd, dtype=torch.float32, device=dev)
    shifted = kv.data_ptr() + 4
    rc, msg = _call(lib, q.data_ptr(), shifted, kv.data_ptr(), H, Hkv, hd, T, 0.088, out.data_ptr(),
                    None)
    assert rc == -1 and "misaligned" in msg
    rc, msg = _call(lib, q.data_ptr(), kv.data_ptr(), shifted, H, Hkv, hd, T, 0.088, out.data_ptr(),
                    None)
    assert rc == -1 and "misaligned" in msg
