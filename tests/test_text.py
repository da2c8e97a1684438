"""The tokenizer and prompt builder (fish_s2pro_b200/text.py), on the CPU.

The reference's tokenizer golden file (tests/fixtures/tokenizer_golden.tsv)
holds ids of the real s2-pro tokenizer.json, which is not available here, so
the BPE restatement (tokenizer_s2cpp.rs) is checked on a synthetic
tokenizer.json of the same shape with hand-derived expectations, and
build_prompt (prompt.rs:105-220) layout by layout.
"""
import json

import numpy as np
import pytest

from fish_s2pro_b200 import PromptCodes, S2dError, S2Tokenizer, build_prompt, load_prompt_codes
from fish_s2pro_b200.text import bytelevel, bytes_to_unicode


def test_byte_level_alphabet():
    t = bytes_to_unicode()
    assert len(set(t.values())) == 256
    assert t[ord("a")] == "a" and t[ord("!")] == "!" and t[0xE9] == "é"
    assert t[ord(" ")] == "Ġ" and t[ord("\n")] == "Ċ"  # the GPT-2 table: space Ġ, newline Ċ
    assert bytelevel("é") == "Ã©"  # UTF-8 bytes C3 A9


def test_bpe_encode(tokenizer_json):
    tok = S2Tokenizer.from_file(tokenizer_json)
    assert (tok.config.im_start_id, tok.config.im_end_id, tok.config.voice_id) == (3000, 4000, 3001)
    # "hello": h e l l o -> he (rank 0) -> ll (1) -> hell (2); o stays
    assert tok.encode_s2cpp("hello") == [258, ord("o")]
    # " world" is one pre-token: Ġ w o r l d -> Ġw (3) -> or (4) -> Ġwor (5)
    assert tok.encode_s2cpp("hello world") == [258, ord("o"), 261, ord("l"), ord("d")]
    # specials split the text; "plain" is an added token that is not special,
    # so it is only found as a whole pre-token in the vocab
    assert tok.encode_s2cpp("<|im_start|>user") == [3000] + [ord(c) for c in "user"]
    assert tok.encode_s2cpp("a<|voice|><|im_end|>plain") == [ord("a"), 3001, 4000, 3003]
    assert tok.encode_s2cpp("plainer") == [ord(c) for c in "plainer"]
    # whitespace starts a new pre-token: "hi", " ", "\n" -> byte symbols Ġ and Ċ (ids 32 and 10)
    assert tok.encode_s2cpp("hi \n") == [ord("h"), ord("i"), 32, 10]
    assert tok.encode_s2cpp("") == []
    assert tok.encode_newline() == [198]
    # multi-byte characters go through their UTF-8 bytes
    assert tok.encode_s2cpp("é") == [0xC3, 0xA9]


def test_tokenizer_errors(tmp_path):
    with pytest.raises(S2dError, match="read tokenizer"):
        S2Tokenizer.from_file(tmp_path / "none.json")
    p = tmp_path / "t.json"
    p.write_text(json.dumps({"added_tokens": [], "model": {"vocab": {"a": 0}, "merges": []}}))
    with pytest.raises(S2dError, match="missing special token"):
        S2Tokenizer.from_file(p)
    p.write_text("{not json")
    with pytest.raises(S2dError, match="parse tokenizer json"):
        S2Tokenizer.from_file(p)


def test_build_prompt_without_reference(tokenizer_json):
    tok = S2Tokenizer.from_file(tokenizer_json)
    p = build_prompt(tok, "hello", 10, 4096)
    data = np.asarray(p.data).reshape(p.rows, p.cols)
    want = ([3000] + tok.encode_s2cpp("user") + [198] + tok.encode_s2cpp("hello") + [4000, 198] + [3000] +
            tok.encode_s2cpp("assistant") + [198, 3001])
    assert p.rows == 11 and list(data[0]) == want and not data[1:].any()
    # an empty reference text (or codes of another codebook count) falls back to this layout
    codes = PromptCodes(10, 3, np.arange(30, dtype=np.uint32))
    assert np.array_equal(build_prompt(tok, "hello", 10, 4096, "", codes).data, p.data)
    assert np.array_equal(build_prompt(tok, "hello", 10, 4096, "x", PromptCodes(9, 3, np.zeros(27))).data, p.data)


def test_build_prompt_with_reference(tokenizer_json):
    tok = S2Tokenizer.from_file(tokenizer_json)
    codes = PromptCodes(10, 3, (np.arange(30, dtype=np.uint32) * 7) % 1024)
    p = build_prompt(tok, "hello", 10, 4096, "ref words", codes)
    data = np.asarray(p.data).reshape(p.rows, p.cols)
    pre = ([3000] + tok.encode_s2cpp("system") + [198] +
           tok.encode_s2cpp("convert the provided text to speech reference to the following:\n\nText:\n") +
           [3002] + tok.encode_s2cpp("ref words") + tok.encode_s2cpp("\n\nSpeech:\n"))
    post = ([4000, 198, 3000] + tok.encode_s2cpp("user") + [198] + tok.encode_s2cpp("hello") + [4000, 198] +
            [3000] + tok.encode_s2cpp("assistant") + [198, 3001])
    c = np.asarray(codes.data).reshape(10, 3)
    assert p.cols == len(pre) + 3 + len(post)
    assert list(data[0, :len(pre)]) == pre and list(data[0, len(pre) + 3:]) == post
    assert list(data[0, len(pre):len(pre) + 3]) == list(c[0] + 4096)
    assert np.array_equal(data[1:, len(pre):len(pre) + 3], c)  # row 1 holds codebook 0 again, unshifted
    assert not data[1:, :len(pre)].any() and not data[1:, len(pre) + 3:].any()
    with pytest.raises(S2dError, match="both be set"):
        build_prompt(tok, "hello", 10, 4096, "ref", None)


def test_load_prompt_codes(tmp_path):
    p = tmp_path / "codes.json"
    p.write_text(json.dumps({"prompt_text": "hi", "num_codebooks": 2, "cols": 3, "codes": [1, 2, 3, 4, 5, 6]}))
    text, codes = load_prompt_codes(p)
    assert text == "hi" and (codes.num_codebooks, codes.cols) == (2, 3) and list(codes.data) == [1, 2, 3, 4, 5, 6]
    p.write_text(json.dumps({"prompt_text": "hi", "num_codebooks": 2, "cols": 3, "codes": [1, 2]}))
    with pytest.raises(S2dError, match="length mismatch"):
        load_prompt_codes(p)


def test_pipeline_load_reports_missing_files(tmp_path, tokenizer_json):
    """pipeline.rs:258 require_file: each of the three files is checked
    before anything is loaded (no GPU needed)."""
    from fish_s2pro_b200 import Pipeline
    lm, codec = tmp_path / "lm.gguf", tmp_path / "codec.gguf"
    with pytest.raises(S2dError, match="transformer GGUF not found"):
        Pipeline.load(lm, codec, tokenizer_json)
    lm.write_bytes(b"GGUF")
    with pytest.raises(S2dError, match="codec GGUF not found"):
        Pipeline.load(lm, codec, tokenizer_json)
    codec.write_bytes(b"GGUF")
    with pytest.raises(S2dError, match="tokenizer not found"):
        Pipeline.load(lm, codec, tmp_path / "tokenizer.json")


def test_synthetic_codec_file_has_the_reference_shapes():
    """The synthetic codec's tensor list: the names and ggml dims the
    reference's loaders check (codec.rs:2386-2413, 860-910, 736-820,
    1640-1679, 1519-1584), and kernel 2 x stride for every strided conv."""
    from fish_s2pro_b200.codec_synth import _tensors
    t = {name: dims for name, dims, _, _ in _tensors()}
    assert t["quantizer.semantic_quantizer.quantizers.0.codebook.weight"] == [8, 4096]
    assert t["quantizer.quantizer.quantizers.8.codebook.weight"] == [8, 1024]
    assert t["quantizer.post_module.layers.7.attention.wqkv.weight"] == [1024, 3072]
    assert t["quantizer.upsample.1.0.conv.weight"] == [2, 1024, 1024]
    assert t["decoder.model.0.conv.weight"] == [7, 1024, 1536]
    assert t["decoder.model.6.conv.weight"] == [7, 96, 1] and t["decoder.model.5.alpha"] == [1, 96, 1]
    for i, (r, c, ci) in enumerate(zip((8, 8, 4, 2), (768, 384, 192, 96), (1536, 768, 384, 192)), start=1):
        assert t[f"decoder.model.{i}.block.1.conv.weight"] == [2 * r, c, ci]
    assert t["encoder.block.0.conv.weight"] == [7, 1, 64] and t["encoder.block.6.conv.weight"] == [3, 1024, 1024]
    for i, (k, c, co) in enumerate(zip((4, 8, 16, 16), (64, 128, 256, 512), (128, 256, 512, 1024)), start=1):
        assert t[f"encoder.block.{i}.block.4.conv.weight"] == [k, c, co]
    assert t["encoder.block.4.block.5.layers.3.feed_forward.w2.weight"] == [3072, 1024]
    assert t["quantizer.downsample.0.0.conv.weight"] == [2, 1024, 1024]
    assert sum(1 for n in t if n.startswith("decoder.")) == 89  # the reference registry's decoder count
