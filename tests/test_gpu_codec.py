"""The codec decode on the GPU (include/s2d_codec.h) against the codec oracle.

* RVQ lookup: bit-exact against a float32 restatement that sums in the
  reference's order (codec.rs:2428-2445, 2580-2588), which the kernel keeps.
* Post module + upsample: within LAT_TOL of the float64 oracle.  The GPU
  feeds float activations to the f16 tensor cores as hi + lo pairs (about
  22 bits) with f32 accumulation; the seeded cases show ~3e-6 of max |ref|.
* Decoder and the whole decode_waveform: the 29 convolutions round their
  inputs to f16 (codec.rs:2257-2259), so any f32-level difference flips the
  odd input to its other f16 neighbour and the stack amplifies it.  The
  oracle run in float32 (the reference's own arithmetic, in another order)
  lands 6e-4 (1 latent frame) to 1.4e-3 (4 frames) of max |ref| away from
  the float64 oracle, and the GPU as far: the decoder bound PCM_TOL is set
  from that spread, and a second test asks that the GPU stay within a small
  multiple of the float32 oracle's own distance.  A wrong tap, channel or
  frame order moves the output by its own magnitude.
* Edge cases from the reference: a single frame, a post-module sequence
  longer than the 128-frame attention window, and every error it raises.
"""
import numpy as np
import pytest

from oracle import codec_oracle as co

pytestmark = pytest.mark.gpu

LAT_TOL = 3e-5
PCM_TOL = 1e-2


@pytest.fixture(scope="module")
def codec(codec_gguf):
    from fish_s2pro_b200 import CodecDecoder
    c = CodecDecoder.open(codec_gguf)
    yield c
    c.close()


def random_codes(n, seed):
    rng = np.random.default_rng(seed)
    return np.concatenate([rng.integers(0, 4096, n), rng.integers(0, 1024, 9 * n)]).astype(np.int32)


def rel_err(got, want):
    return float(np.max(np.abs(np.asarray(got, np.float64) - want)) / np.max(np.abs(want)))


def rvq_f32(codes, n, w):
    """rvq_lookup_codes in float32, each sum left to right (no fused multiply-add)."""
    codes = np.asarray(codes).reshape(10, n)
    lat = np.zeros((n, 1024), np.float32)
    for cb in range(10):
        book, wo, bo = (a.astype(np.float32) for a in w.quantizer(cb))
        for f in range(n):
            row = book[codes[cb, f]]
            p = np.zeros(1024, np.float32)
            for j in range(8):
                p = (p + (wo[:, j] * row[j]).astype(np.float32)).astype(np.float32)
            lat[f] = (lat[f] + (p + bo.astype(np.float32))).astype(np.float32)
    return lat


@pytest.mark.parametrize("n,seed", [(1, 0), (2, 1), (37, 2)])
def test_rvq_lookup_is_bit_exact(codec, codec_oracle_weights, n, seed):
    codes = random_codes(n, seed)
    got = codec.rvq_lookup_codes(codes, 10, n)
    assert got.latents.shape == (n * 1024,) and got.latent_dim == 1024
    assert np.array_equal(got.latents.reshape(n, 1024), rvq_f32(codes, n, codec_oracle_weights))


@pytest.mark.parametrize("n", [1, 2, 5, 33, 136])
def test_decode_latents_matches_oracle(codec, codec_oracle_weights, n):
    """Post module (8 windowed-attention layers; 136 frames cross the
    128-frame window) and the two upsample stages."""
    lat = co.rvq_lookup_codes(random_codes(n, 10 + n), 10, n, codec_oracle_weights)
    got = codec.rvq_decode_latents(lat.astype(np.float32), n)
    assert (got.input_frames, got.output_frames, got.hidden_dim) == (n, 4 * n, 1024)
    want = co.rvq_decode_latents(lat.astype(np.float32).astype(np.float64), codec_oracle_weights)
    assert rel_err(got.hidden.reshape(4 * n, 1024), want) < LAT_TOL


def test_per_frame_attention_route_matches_oracle(codec_gguf, codec_oracle_weights, monkeypatch):
    """S2D_CODEC_ATTN_TILED=0: the windowed attention one block per frame and
    head instead of over 32-frame tiles, across the 128-frame window."""
    from fish_s2pro_b200 import CodecDecoder
    monkeypatch.setenv("S2D_CODEC_ATTN_TILED", "0")
    n = 136
    lat = co.rvq_lookup_codes(random_codes(n, 10 + n), 10, n, codec_oracle_weights)
    with CodecDecoder.open(codec_gguf) as c:
        got = c.rvq_decode_latents(lat.astype(np.float32), n)
    want = co.rvq_decode_latents(lat.astype(np.float32).astype(np.float64), codec_oracle_weights)
    assert rel_err(got.hidden.reshape(4 * n, 1024), want) < LAT_TOL


@pytest.mark.parametrize("L", [1, 4, 9, 33])
def test_decoder_matches_oracle(codec, codec_oracle_weights, L):
    rng = np.random.default_rng(L)
    hidden = rng.standard_normal((L, 1024)).astype(np.float32)
    got = codec.forward_codec_decoder(hidden, L)
    assert got.shape == (512 * L,)
    want = co.forward_codec_decoder(hidden.astype(np.float64), codec_oracle_weights)
    assert rel_err(got, want) < PCM_TOL


def test_im2col_cublas_route_matches_oracle(codec_gguf, codec_oracle_weights, monkeypatch):
    """S2D_CODEC_TC=0: the causal convolutions as im2col + cuBLAS instead of
    the implicit-GEMM tcgen05 kernel, against the same oracle."""
    from fish_s2pro_b200 import CodecDecoder
    monkeypatch.setenv("S2D_CODEC_TC", "0")
    with CodecDecoder.open(codec_gguf) as c:
        rng = np.random.default_rng(4)
        hidden = rng.standard_normal((4, 1024)).astype(np.float32)
        want = co.forward_codec_decoder(hidden.astype(np.float64), codec_oracle_weights)
        assert rel_err(c.forward_codec_decoder(hidden, 4), want) < PCM_TOL


@pytest.mark.parametrize("L", [1, 4])
def test_decoder_is_as_close_as_float32_arithmetic(codec, codec_gguf, codec_oracle_weights, L):
    """The GPU decoder's distance from the float64 oracle is within 3x (plus
    1e-4) of the float32 oracle's own distance from it."""
    w32 = co.CodecWeights(codec_gguf, np.float32)
    rng = np.random.default_rng(100 + L)
    hidden = rng.standard_normal((L, 1024)).astype(np.float32)
    want = co.forward_codec_decoder(hidden.astype(np.float64), codec_oracle_weights)
    e32 = rel_err(co.forward_codec_decoder(hidden, w32), want)
    egpu = rel_err(codec.forward_codec_decoder(hidden, L), want)
    assert egpu < 3 * e32 + 1e-4, (egpu, e32)


def test_fixture_codes_decode_to_the_oracle_waveform(codec, codec_oracle_weights):
    from test_codec_oracle import FIXTURE_CODES
    got = codec.decode_waveform(FIXTURE_CODES, 10, 2)
    assert (got.sample_rate, got.input_frames, got.latent_frames, got.num_samples) == (44100, 2, 8, 4096)
    want = co.decode_waveform(FIXTURE_CODES, 10, 2, codec_oracle_weights)
    assert np.isfinite(got.samples).all() and np.max(np.abs(got.samples)) <= 1.0
    assert rel_err(got.samples, want) < PCM_TOL


def test_decode_is_deterministic_and_the_device_entry_agrees(codec):
    import torch
    codes = random_codes(6, 99)
    a = codec.decode_waveform(codes, 10, 6).samples
    b = codec.decode_waveform(codes, 10, 6).samples
    assert np.array_equal(a, b)
    from fish_s2pro_b200.codec import codec_lib
    cd = torch.from_numpy(codes).cuda()
    out = torch.empty(6 * 2048, dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    assert codec_lib().s2d_codec_decode_waveform_device(codec.handle, cd.data_ptr(), 10, 6, out.data_ptr(),
                                                        s.cuda_stream) == 0
    s.synchronize()
    assert codec_lib().s2d_codec_sync(codec.handle) == 0
    assert np.array_equal(out.cpu().numpy(), a)


def test_wav_bytes(codec):
    from fish_s2pro_b200 import pcm_to_wav
    codes = random_codes(1, 5)
    wav = codec.decode_waveform_to_wav(codes, 10, 1)
    assert wav == pcm_to_wav(codec.decode_waveform(codes, 10, 1).samples)
    assert len(wav) == 44 + 2 * 2048


def test_errors_match_the_reference(codec):
    from fish_s2pro_b200 import S2dError
    codes = random_codes(2, 3)
    with pytest.raises(S2dError, match="codebook count mismatch") as e:
        codec.decode_waveform(codes[:18], 9, 2)
    assert e.value.code == -1
    bad = codes.copy()
    bad[5] = -3
    with pytest.raises(S2dError, match="non-negative"):
        codec.decode_waveform(bad, 10, 2)
    bad = codes.copy()
    bad[2] = 1024  # residual codebook 0 holds 1,024 codes
    with pytest.raises(S2dError, match="out of range"):
        codec.rvq_lookup_codes(bad, 10, 2)
    bad[2] = 0
    bad[0] = 4095  # the semantic codebook holds 4,096
    codec.rvq_lookup_codes(bad, 10, 2)
    with pytest.raises(S2dError, match="at least one frame"):
        codec.decode_waveform(np.zeros(0, np.int32), 10, 0)
    with pytest.raises(S2dError, match="latent dim 1024"):
        codec.forward_codec_decoder(np.zeros(512, np.float32), 1, 512)
    # the device entry flags an out-of-range code for the next sync
    import torch
    from fish_s2pro_b200.codec import codec_lib
    bad = torch.from_numpy(codes.copy()).cuda()
    bad[3] = 5000
    out = torch.empty(2 * 2048, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()  # the codec's own stream does not wait for torch's
    assert codec_lib().s2d_codec_decode_waveform_device(codec.handle, bad.data_ptr(), 10, 2, out.data_ptr(),
                                                        None) == 0
    assert codec_lib().s2d_codec_sync(codec.handle) == -6
    assert codec_lib().s2d_codec_sync(codec.handle) == 0  # the flag is cleared
    # and the codec still decodes
    assert codec.decode_waveform(codes, 10, 2).num_samples == 4096


# ---- reference-audio encoder (codec.rs:1056) ----------------------------------

@pytest.fixture(scope="module")
def w32(codec_gguf):
    return co.CodecWeights(codec_gguf, np.float32)


def pcm(n, seed):
    rng = np.random.default_rng(seed)
    t = np.arange(n)
    return (0.3 * np.sin(t * 0.031) + 0.2 * np.sin(t * 0.0071 + 1.0) + 0.05 * rng.standard_normal(n)).astype(np.float32)


@pytest.mark.parametrize("n", [2048, 5000])
def test_encoder_frontend_matches_oracle(codec, codec_oracle_weights, w32, n):
    """Entry conv, 4 blocks (residual units, strided down convs as two-tap
    implicit GEMMs over rows of stride x C channels), the last block's
    transformer (window 512), tail conv: within 3x (+1e-4) of the float32
    oracle's distance from the float64 oracle, as for the decoder."""
    from test_codec_oracle import fixture_pcm
    audio = fixture_pcm(n) if n == 2048 else pcm(n, 1)
    got = codec.forward_codec_encoder_frontend(audio)
    frames = (n + 2047) // 2048 * 4
    assert (got.input_samples, got.padded_samples, got.output_frames) == (n, frames * 512, frames)
    want, padded = co.forward_codec_encoder_frontend(audio, codec_oracle_weights)
    e32 = rel_err(co.forward_codec_encoder_frontend(audio, w32)[0], want)
    egpu = rel_err(got.hidden.reshape(frames, 1024), want)
    assert egpu < 3 * e32 + 1e-4 and egpu < PCM_TOL, (egpu, e32)


@pytest.mark.parametrize("n", [8, 16])
def test_quantizer_encode_stage_matches_oracle(codec, codec_oracle_weights, w32, n):
    """Two stride-2 downsample stages (one-tap implicit GEMMs over rows of
    2 x 1024) with their ConvNeXt blocks, and the 8-layer pre module; the
    8-frame input is the reference fixture's (codec.rs:4107-4110)."""
    if n == 8:
        lat = (((np.arange(8 * 1024) % 97) - 48.0) / 512.0).reshape(8, 1024).astype(np.float32)
    else:
        lat = np.random.default_rng(n).standard_normal((n, 1024)).astype(np.float32)
    got = codec.forward_codec_quantizer_encode_stage(lat, n)
    assert (got.input_frames, got.output_frames) == (n, n // 4)
    want = co.forward_codec_quantizer_encode_stage(lat.astype(np.float64), codec_oracle_weights)
    e32 = rel_err(co.forward_codec_quantizer_encode_stage(lat, w32), want)
    egpu = rel_err(got.hidden.reshape(n // 4, 1024), want)
    assert egpu < 3 * e32 + 1e-5 and egpu < 1e-3, (egpu, e32)


def test_vq_encode_matches_oracle(codec, codec_oracle_weights):
    """Nearest-code search: per frame the codes equal the oracle's in order;
    a codebook may differ only where the oracle's best two cosine scores are
    within 1e-4 (a near tie), after which the frame's later codebooks follow
    a different residual and are not compared."""
    n = 24
    lat = co.forward_codec_quantizer_encode_stage(
        np.random.default_rng(5).standard_normal((4 * n, 1024)), codec_oracle_weights)
    got = codec.rvq_encode_latents_nearest(lat.astype(np.float32), n)
    want, l2, gaps = co.rvq_encode_latents_nearest(lat.astype(np.float32).astype(np.float64), codec_oracle_weights,
                                                   margins=True)
    gc = got.codes.reshape(10, n)
    exact = 0
    for f in range(n):
        same = True
        for cb in range(10):
            if gc[cb, f] != want[cb, f]:
                assert gaps[cb, f] < 1e-4, (f, cb, gaps[cb, f])
                same = False
                break
        if same:
            exact += 1
            assert abs(got.final_residual_l2[f] - l2[f]) <= 1e-5 * l2[f]
    assert exact >= n - 2


def test_encode_reference_audio_chains_the_stages(codec, tmp_path):
    """The one-call encode equals its three stages run one by one, its codes
    are in range, decode back to 2,048 samples a frame, and the WAV entry
    reads the file as the reference does."""
    from fish_s2pro_b200.codec import pcm_to_wav
    audio = pcm(4500, 3)
    r = codec.encode_reference_audio(audio)
    assert (r.input_samples, r.padded_samples, r.encoder_frames, r.quantizer_frames) == (4500, 6144, 12, 3)
    fe = codec.forward_codec_encoder_frontend(audio)
    q = codec.forward_codec_quantizer_encode_stage(fe.hidden, fe.output_frames)
    v = codec.rvq_encode_latents_nearest(q.hidden, q.output_frames)
    assert np.array_equal(r.codes, v.codes) and np.array_equal(r.final_residual_l2, v.final_residual_l2)
    codes = r.codes.reshape(10, 3)
    assert (0 <= codes[0]).all() and (codes[0] < 4096).all() and (0 <= codes[1:]).all() and (codes[1:] < 1024).all()
    assert codec.decode_waveform(r.codes, 10, 3).num_samples == 3 * 2048
    wav = tmp_path / "ref.wav"
    wav.write_bytes(pcm_to_wav(audio))
    from fish_s2pro_b200 import read_wav_mono_f32
    assert np.array_equal(codec.encode_reference_wav_file(wav).codes,
                          codec.encode_reference_audio(read_wav_mono_f32(wav)).codes)


def test_encoder_edge_cases(codec):
    from fish_s2pro_b200 import S2dError
    assert codec.has_encoder
    r = codec.encode_reference_audio(np.zeros(0, np.float32))  # no samples: one padded frame
    assert (r.padded_samples, r.quantizer_frames) == (2048, 1) and r.codes.size == 10
    with pytest.raises(S2dError, match="multiple of 4"):
        codec.forward_codec_quantizer_encode_stage(np.zeros(6 * 1024, np.float32), 6)


def test_decode_is_causal_at_full_size(codec):
    """A size-independent property at the bench's scale: every stage is causal
    (left-padded convolutions, windowed causal attention, transposed
    convolutions that write forward), so the first k frames' samples of a
    512-frame decode (multi-wave convolution grids, sliced GEMMs) equal the
    decode of those k frames alone, which the oracle tests pin, up to the
    f32-level spread of the f16-rounded stack."""
    codes = random_codes(512, 77).reshape(10, 512)
    full = codec.decode_waveform(codes.reshape(-1), 10, 512).samples
    for k in (3, 40):
        head = codec.decode_waveform(np.ascontiguousarray(codes[:, :k]).reshape(-1), 10, k).samples
        assert rel_err(full[:k * 2048], head.astype(np.float64)) < PCM_TOL, k
    # and the rows past the first k do depend on the later codes
    other = codes.copy()
    other[:, 40:] = random_codes(472, 78).reshape(10, 472)
    alt = codec.decode_waveform(other.reshape(-1), 10, 512).samples
    assert rel_err(alt[:40 * 2048], full[:40 * 2048].astype(np.float64)) < PCM_TOL
    assert np.max(np.abs(alt[41 * 2048:] - full[41 * 2048:])) > 1e-2


def test_encode_is_causal_at_full_size(codec):
    """The encoder is causal too, so the first frames' codes of a 10 s clip
    (the bench's size) match the encode of the clip's first 4 frames of
    samples; a code may differ only by a near tie of the nearest-code search
    after f32-level differences, so at least 95% must agree."""
    audio = pcm(441000, 9)
    full = codec.encode_reference_audio(audio).codes.reshape(10, -1)
    head = codec.encode_reference_audio(audio[:4 * 2048]).codes.reshape(10, 4)
    assert full.shape == (10, 216)
    assert np.mean(full[:, :4] == head) >= 0.95
