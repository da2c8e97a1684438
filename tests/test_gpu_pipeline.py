"""Text (+ reference voice) -> speech through fish_s2pro_b200.Pipeline
(pipeline.rs:127-256): prompt building, the persistent-engine code
generation, the codec decode and the WAV bytes, on a tiny Dual-AR whose 10
codebooks the synthetic s2-pro codec decodes, with a synthetic
tokenizer.json.  Each stage has its own parity tests; these check that the
pipeline wires them as the reference does.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FRAMES = 6


@pytest.fixture(scope="module")
def pipe(model_dir, codec_gguf, tokenizer_json):
    from fish_s2pro_b200 import Pipeline, configs, synth
    lm = synth.cached_gguf(configs.tiny_codec(), model_dir)
    p = Pipeline.load(lm, codec_gguf, tokenizer_json, max_seq_len=512)
    yield p
    p.close()


def params():
    from fish_s2pro_b200 import GenerateParams
    return GenerateParams(FRAMES, 0.0, 1.0, 0, 2 * FRAMES + 2)


def test_synthesize_without_reference(pipe):
    from fish_s2pro_b200 import SeededRng, SynthesisOptions, build_prompt, generate_codes
    r = pipe.synthesize(SynthesisOptions("hello world", params=params(), seed=3))
    assert r.codes.n_frames == FRAMES and r.codes.num_codebooks == 10
    assert r.waveform.num_samples == FRAMES * 2048 and r.waveform.sample_rate == 44100
    assert len(r.wav_bytes) == 44 + 2 * FRAMES * 2048
    prompt = build_prompt(pipe.tokenizer, "hello world", 10, pipe.graph.semantic_begin_id)
    assert r.prompt_cols == prompt.cols
    # the same as the stages called one by one
    codes = generate_codes(pipe.state, pipe.tokenizer.config, pipe.graph, prompt, params(), pipe.fast, SeededRng(3))
    assert np.array_equal(codes.codes, r.codes.codes)
    assert np.array_equal(pipe.codec.decode_waveform(codes.codes, 10, FRAMES).samples, r.waveform.samples)
    # and deterministic for the seed (the cached prompt is reused)
    assert np.array_equal(pipe.synthesize(SynthesisOptions("hello world", params=params(), seed=3)).codes.codes,
                          r.codes.codes)


def test_synthesize_with_a_reference_voice(pipe, tmp_path):
    from fish_s2pro_b200 import S2dError, SynthesisOptions, build_prompt, pcm_to_wav
    t = np.arange(44100)
    wav = tmp_path / "voice.wav"
    wav.write_bytes(pcm_to_wav((0.3 * np.sin(t * 0.05) + 0.1 * np.sin(t * 0.013)).astype(np.float32)))
    ref = pipe.encode_reference_wav(wav)
    assert (ref.num_codebooks, ref.cols) == (10, 22)  # ceil(44,100 / 2,048) frames
    o = SynthesisOptions("hello world", prompt_text="ref words", prompt_codes=ref, params=params(), seed=5)
    r = pipe.synthesize(o)
    prompt = build_prompt(pipe.tokenizer, "hello world", 10, pipe.graph.semantic_begin_id, "ref words", ref)
    assert r.prompt_cols == prompt.cols and r.codes.n_frames == FRAMES
    assert r.waveform.num_samples == FRAMES * 2048 and np.isfinite(r.waveform.samples).all()
    with pytest.raises(S2dError, match="both be set"):
        pipe.synthesize(SynthesisOptions("hello", prompt_text="ref words", params=params()))
