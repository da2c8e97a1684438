"""Pin the CPU oracle against the reference's own known-answer tests.

Every expected value below is transcribed from a unit test of the reference
(crate fish_s2_infer / fish_s2_core; the test is cited beside each case).  The
reference is Rust and cannot be built here, so these known answers are what
anchors the oracle to it.
"""
import math
import struct

import numpy as np
import pytest

from oracle import oracle as o

F32 = np.float32


def close(actual, expected, tol):
    actual = np.asarray(actual, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    assert actual.shape == expected.shape
    assert np.all(np.abs(actual - expected) < tol), (actual, expected)


# ---- tensor.rs ------------------------------------------------------------

def test_decodes_f16_le_bytes_to_f32_values():  # tensor.rs:338-345
    vals = [o.f16_to_f32(b) for b in (0x3C00, 0xC000, 0x3800, 0x4400)]
    assert vals == [1.0, -2.0, 0.5, 4.0]


def test_rounds_f32_to_f16_values():  # tensor.rs:356-364
    assert o.round_f32_to_f16(1.0) == 1.0
    assert o.round_f32_to_f16(-2.0) == -2.0
    assert o.round_f32_to_f16(0.5) == 0.5
    assert o.f32_to_f16(math.inf) == 0x7C00
    assert o.f32_to_f16(-math.inf) == 0xFC00
    assert o.f32_to_f16(math.nan) & 0x7C00 == 0x7C00


def test_f16_decode_matches_ieee_for_every_non_nan_pattern():
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    ours = np.array([o.f16_to_f32(int(b)) for b in bits], dtype=F32)
    finite = ~np.isnan(ref)
    assert np.array_equal(ours[finite].view(np.uint32), ref[finite].view(np.uint32))


def test_f32_to_f16_rounds_to_nearest_even_like_ieee():
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.standard_normal(4000).astype(F32) * 10,
                         rng.uniform(-7e-5, 7e-5, 2000).astype(F32),
                         np.array([65504, 65520, 65519.99, 6.1e-5, 5.96e-8, 2.98e-8], F32)])
    ours = np.array([o.f32_to_f16(float(x)) for x in xs], dtype=np.uint16)
    assert np.array_equal(ours, xs.astype(np.float16).view(np.uint16))


def test_rms_norm_matches_manual_smoke():  # tensor.rs:366-371
    out = o.rms_norm([1.0, 2.0, 3.0, 4.0], [1.0, 0.5, 2.0, -1.0], 1e-6)
    scale = F32(1.0) / np.sqrt(F32(7.5) + F32(1e-6))
    close(out, [scale, scale, 6.0 * scale, -4.0 * scale], 1e-6)


def test_linear_matches_ggml_output_input_weight_layout():  # tensor.rs:373-377, backend.rs:207-215
    out = o.linear([2.0, -1.0], [1.0, 2.0, 3.0, 4.0, 5.0, 6.0], 2, 3)
    assert list(out) == [0.0, 2.0, 4.0]


def test_linear_rejects_bad_weight_shape():  # backend.rs:217-223
    with pytest.raises(o.OracleError, match="linear weight length mismatch"):
        o.linear([1.0, 2.0], [1.0, 2.0, 3.0], 2, 2)


def test_matvec_f16_streaming_matches_expanded_linear():  # tensor.rs:379-391
    w = [o.f32_to_f16(v) for v in (1.0, 2.0, 3.0, 4.0, 5.0, 6.0)]
    close(o.matvec_f16([2.0, -1.0], w, 2, 3), [0.0, 2.0, 4.0], 1e-6)


def test_rms_norm_rejects_empty_and_mismatch():  # backend.rs:84-94
    with pytest.raises(o.OracleError, match="empty"):
        o.rms_norm([], [], 1e-6)
    with pytest.raises(o.OracleError, match="length mismatch"):
        o.rms_norm([1.0, 2.0], [1.0], 1e-6)


# ---- attention.rs ----------------------------------------------------------

def test_rope_normal_rotates_adjacent_pairs():  # attention.rs:336-343
    out = o.rope_normal([1.0, 0.0, 0.0, 1.0], 4, 1, 10_000.0)
    s1, c1 = math.sin(1.0), math.cos(1.0)
    s2, c2 = math.sin(0.01), math.cos(0.01)
    close(out, [c1, s1, -s2, c2], 1e-5)


def test_rope_rejects_odd_head_dim():  # attention.rs:178-182
    with pytest.raises(o.OracleError, match="non-zero and even"):
        o.rope_normal([1.0, 2.0, 3.0], 3, 0, 10_000.0)


def test_kv_cache_uses_s2_layout_for_token_writes():  # attention.rs:345-360
    kv = o.KvCache(2, 2, 3, 2)
    kv.write_token(1, 2, [1, 2, 3, 4], [5, 6, 7, 8])
    k, v = kv.read_token(1, 2)
    assert list(k) == [1, 2, 3, 4] and list(v) == [5, 6, 7, 8]
    with pytest.raises(o.OracleError, match="out of bounds"):
        kv.write_token(2, 0, [0] * 4, [0] * 4)


def test_gqa_decode_attention_repeats_kv_heads():  # attention.rs:362-406
    q = [1, 0, 0, 1, 1, 0, 0, 1]
    keys = [1, 0, 0, 1, 0, 1, 1, 0]
    vals = [10, 0, 0, 10, 20, 0, 0, 20]
    out = o.gqa_decode_attention(q, keys, vals, 4, 2, 2, 2, 1.0)
    p_hi = math.exp(1) / (math.exp(1) + 1.0)
    p_lo = 1.0 - p_hi
    close(out, [10 * p_hi + 20 * p_lo, 0.0, 10 * p_lo + 20 * p_hi, 0.0,
                0.0, 10 * p_lo + 20 * p_hi, 0.0, 10 * p_hi + 20 * p_lo], 1e-5)


def test_decode_attention_reads_written_kv_cache():  # attention.rs:408-428
    kv = o.KvCache(2, 1, 2, 1)
    kv.write_token(0, 0, [1, 0], [2, 0])
    kv.write_token(0, 1, [0, 1], [4, 0])
    out = kv.decode_attention(0, 2, [1, 0, 0, 1], 2, 1.0)
    p_hi = math.exp(1) / (math.exp(1) + 1.0)
    p_lo = 1.0 - p_hi
    close(out, [2 * p_hi + 4 * p_lo, 0.0, 2 * p_lo + 4 * p_hi, 0.0], 1e-5)


# ---- slow_ar.rs toy layer ---------------------------------------------------

TOY_SHAPE = dict(hidden_size=4, feed_forward_size=2, head_count=2, head_count_kv=1, head_dim=2,
                 rope_base=10_000.0, rms_norm_eps=0.0)


def toy_weights():  # slow_ar.rs:1664-1698
    r = math.sqrt(0.5)
    wqkv = [[1, 0, 0, 0], [0] * 4, [0] * 4, [1, 0, 0, 0], [1, 0, 0, 0], [0] * 4,
            [3, 0, 0, 0], [0] * 4]
    wo = [[1, 0, 0, 0], [0, 0, 2, 0], [0] * 4, [0] * 4]
    return dict(attention_norm=[0.5, 1, 1, 1], q_norm=[r, r], k_norm=[r, r],
                wqkv=np.array(wqkv, F32).ravel(), wo=np.array(wo, F32).ravel(),
                ffn_norm=[1.0] * 4, w1=[0.0] * 8, w2=[0.0] * 8, w3=[0.0] * 8)


def test_slow_ar_layer_skeleton_runs_single_token_decode_flow():  # slow_ar.rs:1282-1349
    kv = o.KvCache(2, 1, 1, 1)
    hidden, tr = o.layer_forward(TOY_SHAPE, toy_weights(), [1.0, 0, 0, 0], kv,
                                 decode_loop=True)
    close(tr["normalized"][0], [1, 0, 0, 0], 1e-5)
    close(tr["query"][0], [1, 0, 0, 1], 1e-5)
    close(tr["key"][0], [1, 0], 1e-5)
    close(tr["value"][0], [3, 0], 1e-5)
    k, v = kv.read_token(0, 0)
    close(k, [1, 0], 1e-5)
    close(v, [3, 0], 1e-5)
    close(tr["attention"][0], [3, 0, 3, 0], 1e-5)
    close(tr["projected"][0], [3, 6, 0, 0], 1e-5)
    close(tr["attn_hidden"][0], [4, 6, 0, 0], 1e-5)


def test_slow_ar_layer_skeleton_runs_multi_token_decode_sequence():  # slow_ar.rs:1454-1493
    tokens = np.array([[1, 0, 0, 0], [1, 1, 0, 0]], F32)
    kv_a, kv_b = o.KvCache(2, 1, 2, 1), o.KvCache(2, 1, 2, 1)
    ha, ta = o.layer_forward(TOY_SHAPE, toy_weights(), tokens, kv_a, decode_loop=True)
    hb, tb = o.layer_forward(TOY_SHAPE, toy_weights(), tokens, kv_b, decode_loop=False)
    for k in ta:  # prefill_outputs == outputs, bit for bit
        assert np.array_equal(ta[k], tb[k]), k
    assert np.array_equal(kv_a.read_token(0, 1)[1], kv_b.read_token(0, 1)[1])
    assert np.all(np.isfinite(ta["attention"][1])) and np.all(np.isfinite(ta["attn_hidden"][1]))
    assert not np.array_equal(ta["attn_hidden"][0], ta["attn_hidden"][1])


def test_slow_ar_layer_skeleton_runs_block_prefill_with_ffn_residual():  # slow_ar.rs:1495-1515
    kv = o.KvCache(2, 1, 1, 1)
    hidden, tr = o.layer_forward(TOY_SHAPE, toy_weights(), [1.0, 0, 0, 0], kv)
    close(tr["attn_hidden"][0], [4, 6, 0, 0], 1e-5)
    close(tr["ffn_projected"][0], [0, 0, 0, 0], 1e-5)
    close(hidden, tr["attn_hidden"][0], 1e-5)


def test_swiglu_split_applies_silu_gate():  # slow_ar.rs:1517-1521
    close(o.swiglu_slow([0.0, 1.0], [2.0, 3.0]), [0.0, 3.0 / (1.0 + math.exp(-1.0))], 1e-5)
    close(o.swiglu_fast([0.0, 1.0], [2.0, 3.0]), [0.0, 3.0 / (1.0 + math.exp(-1.0))], 1e-5)


def test_slow_ar_layer_skeleton_rejects_bad_weight_shapes():  # slow_ar.rs:1523-1554
    w = toy_weights()
    w["wqkv"] = [0.0] * 3
    w["q_norm"] = [1.0, 1.0]
    w["k_norm"] = [1.0, 1.0]
    kv = o.KvCache(2, 1, 1, 1)
    with pytest.raises(o.OracleError, match="wqkv_weight length mismatch"):
        o.layer_forward(TOY_SHAPE, w, [0.0] * 4, kv, decode_loop=True)


# ---- sampling.rs ------------------------------------------------------------

def test_semantic_mask_leaves_only_allowed_ids_finite():  # sampling.rs:247-256
    lg = o.semantic_mask_logits([1, 2, 3, 4, 5], 1, 2, 4, False)
    assert lg[0] == -math.inf and lg[1] == 2 and lg[2] == 3 and lg[3] == -math.inf and lg[4] == 5


def test_semantic_mask_can_block_im_end():  # sampling.rs:258-263
    lg = o.semantic_mask_logits([0.1, 0.2, 0.3, 0.4, 0.5], 1, 2, 4, True)
    assert lg[4] == -math.inf


def test_apply_semantic_bias_zeros_disallowed_logits():  # sampling.rs:265-274
    bias = o.build_semantic_bias(5, 1, 2, 4)
    lg = o.apply_semantic_bias([0.1, 0.2, 0.3, 0.4, 0.5], bias, False, 4)
    assert lg[0] == -math.inf and lg[1] == F32(0.2) and lg[4] == F32(0.5)


def test_greedy_temp_zero_picks_top_logit():  # sampling.rs:276-287
    assert o.sample_token([0.1, 5.0, 3.0, 2.0], 0.0, 1.0, 0, None, o.SeededRng(1)) == 1


def test_top_k_limits_candidates():  # sampling.rs:289-300
    assert o.sample_token([10.0, 9.0, 8.0, 0.0], 0.0, 1.0, 2, None, o.SeededRng(99)) <= 1


def test_always_include_id_survives_top_k_truncation():  # sampling.rs:302-313
    lg = [-math.inf] * 4 + [5.0]
    assert o.sample_token(lg, 0.0, 1.0, 1, 4, o.SeededRng(1)) == 4


def test_seeded_sampling_is_repeatable():  # sampling.rs:315-328
    lg = [1.0, 3.0, 2.0, 0.5, 4.0]
    a = o.sample_token(lg, 0.8, 0.9, 3, None, o.SeededRng(42))
    b = o.sample_token(lg, 0.8, 0.9, 3, None, o.SeededRng(42))
    assert a == b


def test_seeded_rng_lcg_sequence():  # sampling.rs:46-52
    rng = o.SeededRng(7)
    state = 7
    for _ in range(8):
        state = (state * 6364136223846793005 + 1) & 0xFFFFFFFFFFFFFFFF
        want = ((state >> 11) & ((1 << 53) - 1)) / float(1 << 53)
        assert rng.next_unit() == want


# ---- generate.rs / prompt.rs -------------------------------------------------

def test_compact_codes_trims_stride_when_fewer_frames():  # generate.rs:409-415
    codes = np.array([10, 11, 0, 20, 21, 0], dtype=np.int32)
    n = o.ctypes.c_int64()
    o._check(o.lib().s2o_compact_codes(o._p(codes, o.ctypes.c_int32), 2, 3, 2, o.ctypes.byref(n)))
    assert list(codes[: n.value]) == [10, 11, 20, 21]


def test_transpose_matches_time_major_layout():  # prompt.rs:288-303
    data = np.array([10, 20, 1, 2, 3, 4], dtype=np.uint32)
    flat = np.empty(6, dtype=np.int32)
    o._check(o.lib().s2o_transpose_to_time_major(o._p(data, o.ctypes.c_uint32), 3, 2,
                                                 o._p(flat, o.ctypes.c_int32)))
    assert list(flat) == [10, 1, 3, 20, 2, 4]


# ---- gguf.rs -----------------------------------------------------------------

def write_tiny_gguf(path):  # gguf.rs:678-705
    b = bytearray(b"GGUF")
    b += struct.pack("<IQQ", 3, 1, 1)

    def s(x):
        return struct.pack("<Q", len(x)) + x.encode()

    b += s("general.architecture") + struct.pack("<I", 8) + s("s2-pro-test")
    b += s("blk.0.weight") + struct.pack("<IQQIQ", 2, 2, 2, 0, 0)
    b += b"\0" * ((32 - len(b) % 32) % 32)
    b += struct.pack("<4f", 1.0, 2.0, 3.0, 4.0)
    path.write_bytes(bytes(b))


def test_reads_tensor_directory_and_bytes(tmp_path):  # gguf.rs:519-558
    p = tmp_path / "tiny.gguf"
    write_tiny_gguf(p)
    g = o.Gguf(p)
    assert g.version == 3 and g.data_start % 32 == 0
    ts = g.tensors()
    assert [t["name"] for t in ts] == ["blk.0.weight"]
    assert ts[0]["dims"] == [2, 2] and ts[0]["type"] == 0 and ts[0]["rel_offset"] == 0
    assert ts[0]["bytes"] == 16
    assert np.frombuffer(g.tensor_bytes("blk.0.weight"), "<f4").tolist() == [1, 2, 3, 4]
    assert g.metadata("general.architecture") == "s2-pro-test"


def test_rejects_non_gguf(tmp_path):  # gguf.rs:510-517
    p = tmp_path / "bad.bin"
    p.write_bytes(b"notgguf")
    with pytest.raises(o.OracleError, match="not a GGUF"):
        o.Gguf(p)


def test_rejects_truncated_tensor(tmp_path):  # gguf.rs:343-362
    p = tmp_path / "trunc.gguf"
    write_tiny_gguf(p)
    p.write_bytes(p.read_bytes()[:-4])
    with pytest.raises(o.OracleError, match="extends past file end"):
        o.Gguf(p)
