"""fish_s2pro_b200 -- sm_100a Dual-AR token loop for fish-s2pro.

The product is libs2d.so (C ABI: include/s2d.h).  This package holds its
sources (csrc/), the in-tree build (build.py), the Python mirror of the
reference's `rust-pure` interface (s2d.py), the workload configurations
(configs.py), the seeded synthetic GGUF writers (synth.py, codec_synth.py),
the continuous-batching scheduler over the s2d_serve_* calls (serve.py),
the codec from codes to PCM and from reference audio to prompt codes
(codec.py, include/s2d_codec.h), the tokenizer and prompt builder (text.py)
and the text-to-speech pipeline over all of it (pipeline.py).
"""
from .s2d import (  # noqa: F401
    LOGITS_ALLOWED,
    LOGITS_FULL,
    LOGITS_NONE,
    CudaMatmulBackend,
    DecodeProfile,
    FastArWeights,
    GenerateCodesResult,
    GenerateParams,
    GraphSpec,
    PromptTensor,
    S2dError,
    SamplerParams,
    SeededRng,
    SlowArState,
    SlowArStepResult,
    forward_codebook_prefix,
    generate_codebooks_for_semantic,
    generate_codes,
    generate_codes_batch,
    RNG_PHILOX,
    RNG_SEEDED,
    lib,
    nccl_unique_id,
    tp_plan,
    sample_token,
    transpose_to_time_major,
)
from .serve import ServeSession, TtsScheduler  # noqa: F401,E402
from .codec import Codec, CodecDecoder, CodecWaveformResult, pcm_to_wav, read_wav_mono_f32  # noqa: F401,E402
from .text import PromptCodes, S2Tokenizer, build_prompt, load_prompt_codes  # noqa: F401,E402
from .pipeline import Pipeline, SynthesisOptions, SynthesisResult  # noqa: F401,E402
