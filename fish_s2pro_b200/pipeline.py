"""Text (+ reference voice) -> speech, end to end: the reference's
`RustPipeline` (crates/fish_s2_infer/src/pipeline.rs:28-260) over this
package's GPU calls.

`Pipeline.load` opens the transformer GGUF (the persistent-engine Dual-AR
state), the codec GGUF (decode and reference-audio encode) and the
tokenizer.json; `synthesize` builds the prompt (cached for repeated
requests, pipeline.rs:199-229), generates the codes with the reference's
SeededRng, decodes them to PCM and writes the WAV bytes;
`encode_reference_wav` turns a voice clip into prompt codes.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from pathlib import Path
from typing import Optional

import numpy as np

from .codec import Codec, CodecWaveformResult, pcm_to_wav
from .s2d import (FastArWeights, GenerateCodesResult, GenerateParams, S2dError, SeededRng, SlowArState,
                  generate_codes)
from .text import PromptCodes, S2Tokenizer, build_prompt


@dataclass
class SynthesisOptions:  # pipeline.rs:57-96
    text: str
    prompt_text: Optional[str] = None
    prompt_codes: Optional[PromptCodes] = None
    params: GenerateParams = field(default_factory=GenerateParams)
    seed: int = 0


@dataclass
class SynthesisResult:  # pipeline.rs:98-103
    prompt_cols: int
    codes: GenerateCodesResult
    waveform: CodecWaveformResult
    wav_bytes: bytes


def _require_file(kind: str, path) -> None:
    """pipeline.rs:258: a clear error before any loading starts."""
    if not Path(path).is_file():
        raise S2dError(-2, f"{kind} not found: {path}")


class Pipeline:
    def __init__(self, state: SlowArState, codec: Codec, tokenizer: S2Tokenizer):
        self.state = state
        self.codec = codec
        self.tokenizer = tokenizer
        self.graph = state.graph_spec()
        self.fast = FastArWeights.from_state(state)
        self._cache = None

    @classmethod
    def load(cls, transformer_gguf, codec_gguf, tokenizer_path, max_seq_len: Optional[int] = None,
             device: int = 0) -> "Pipeline":
        """pipeline.rs:127-164."""
        _require_file("transformer GGUF", transformer_gguf)
        _require_file("codec GGUF", codec_gguf)
        _require_file("tokenizer", tokenizer_path)
        tok = S2Tokenizer.from_file(tokenizer_path)
        state = SlowArState.open(transformer_gguf, max_seq_len=max_seq_len or 32768, device=device)
        try:
            codec = Codec.open(codec_gguf, device=device)
        except Exception:
            state.close()
            raise
        return cls(state, codec, tok)

    def close(self) -> None:
        self.codec.close()
        self.state.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def graph_spec(self):
        return self.graph

    def _prompt(self, o: SynthesisOptions):
        key = (o.text, o.prompt_text, None if o.prompt_codes is None else
               (o.prompt_codes.num_codebooks, o.prompt_codes.cols, np.asarray(o.prompt_codes.data).tobytes()))
        if self._cache is not None and self._cache[0] == key:
            return self._cache[1]
        p = build_prompt(self.tokenizer, o.text, self.graph.num_codebooks, self.graph.semantic_begin_id,
                         o.prompt_text, o.prompt_codes)
        self._cache = (key, p)
        return p

    def synthesize(self, options: SynthesisOptions) -> SynthesisResult:
        """pipeline.rs:166-197: prompt -> generate_codes (SeededRng(seed))
        -> decode_waveform -> pcm_to_wav."""
        if (options.prompt_text is None) != (options.prompt_codes is None):
            raise S2dError(-1, "prompt_text and prompt_codes must both be set or both omitted")
        prompt = self._prompt(options)
        codes = generate_codes(self.state, self.tokenizer.config, self.graph, prompt, options.params, self.fast,
                               SeededRng(options.seed))
        wave = self.codec.decode_waveform(codes.codes[:codes.num_codebooks * codes.n_frames], codes.num_codebooks,
                                          codes.n_frames)
        return SynthesisResult(prompt.cols, codes, wave, pcm_to_wav(wave.samples, wave.sample_rate))

    def encode_reference_wav(self, path) -> PromptCodes:
        """pipeline.rs:235-256."""
        r = self.codec.encode_reference_wav_file(path)
        if r.codes.size != r.quantizer_frames * r.num_codebooks:
            raise S2dError(-1, f"reference prompt codes length mismatch: expected "
                               f"{r.quantizer_frames * r.num_codebooks}, got {r.codes.size}")
        if (r.codes < 0).any():
            raise S2dError(-1, f"reference codebook id is negative: {int(r.codes.min())}")
        return PromptCodes(r.num_codebooks, r.quantizer_frames, r.codes.astype(np.uint32))
