"""The five workload configurations of the Dual-AR benchmark (C1..C5).

Shapes follow the reference's transformer registry
(crates/fish_s2_infer/src/registry.rs:8-28 and
docs/S2_PRO_TRANSFORMER_REGISTRY.md:56-73).  No real weights or prompts are
available offline: every configuration is a seeded random-init model and a
seeded synthetic prompt with the stated shapes and value distributions.

Deviation: the reference feeds the Slow-AR hidden straight into the Fast-AR
(crates/fish_s2_infer/src/fast_ar.rs:393-394) and rejects `fast_project_in`,
so the Fast-AR hidden size equals the Slow-AR one in every configuration
(C1's Fast-AR uses d = 512 instead of 256; C2..C5 use the registry's 2560).
"""
from __future__ import annotations

import dataclasses

import numpy as np

GGML_F16, GGML_Q8_0, GGML_Q4_K = 1, 8, 12


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    name: str
    slow_layers: int
    d: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    sem_begin: int
    sem_end: int
    fast_layers: int
    fast_heads: int
    fast_kv_heads: int
    fast_head_dim: int
    fast_ffn: int
    num_codebooks: int
    codebook_size: int
    context_length: int
    linear_type: int = GGML_F16
    rope_base: float = 1_000_000.0
    eps: float = 1e-6
    weight_std: float = 0.02
    seed: int = 0

    @property
    def fast_context_length(self) -> int:
        return self.num_codebooks + 1


@dataclasses.dataclass(frozen=True)
class Workload:
    """A model plus the decode job the benchmark runs on it."""

    model: ModelConfig
    prompt_len: int
    frames: int
    prompt_seed: int
    im_end_id: int
    batch: int = 1
    prompt_len_min: int = 0  # batch > 1: prompt lengths uniform in [prompt_len_min, prompt_len]

    def prompt(self) -> np.ndarray:
        """Row-major (num_codebooks+1) x prompt_len prompt (PromptTensor,
        prompt.rs:59-67): row 0 holds text ids uniform over the text vocabulary
        (ids below sem_begin), codebook rows are 0 for text positions."""
        rng = np.random.default_rng(self.prompt_seed)
        m = self.model
        p = np.zeros((m.num_codebooks + 1, self.prompt_len), dtype=np.uint32)
        p[0] = rng.integers(0, m.sem_begin, size=self.prompt_len, dtype=np.uint32)
        return p

    def batch_prompts(self) -> list:
        """The `batch` prompts of a batched workload: lengths uniform in
        [prompt_len_min, prompt_len] and text ids uniform over the text
        vocabulary, both from prompt_seed; codebook rows 0."""
        rng = np.random.default_rng(self.prompt_seed)
        m = self.model
        lo = self.prompt_len_min or self.prompt_len
        lens = rng.integers(lo, self.prompt_len + 1, size=self.batch)
        out = []
        for n in lens:
            p = np.zeros((m.num_codebooks + 1, int(n)), dtype=np.uint32)
            p[0] = rng.integers(0, m.sem_begin, size=int(n), dtype=np.uint32)
            out.append(p)
        return out

    def gen_params(self, greedy: bool = True) -> dict:
        """Greedy decoding as in the reference's own greedy tests
        (generate.rs:466-471); im_end blocked for the whole run so that every
        run emits exactly `frames` frames (the block test compares
        2*step_index with min_tokens_before_end, generate.rs:198-201)."""
        if greedy:
            return dict(max_new_tokens=self.frames, temperature=0.0, top_p=1.0, top_k=0,
                        min_tokens_before_end=2 * self.frames + 2, im_end_id=self.im_end_id)
        return dict(max_new_tokens=self.frames, temperature=0.8, top_p=0.9, top_k=30,
                    min_tokens_before_end=2 * self.frames + 2, im_end_id=self.im_end_id)


def tiny(seed: int = 0, linear_type: int = GGML_F16) -> ModelConfig:
    """C1: 4 Slow-AR layers, d 512, 8/2 heads x 64, FFN 1536, 4096 text +
    1024 semantic ids; Fast-AR 2 layers (d 512), 4/2 heads x 64, FFN 768,
    4 codebooks x 1024."""
    return ModelConfig(name="tiny", slow_layers=4, d=512, heads=8, kv_heads=2, head_dim=64,
                       ffn=1536, vocab=5120, sem_begin=4096, sem_end=5119, fast_layers=2,
                       fast_heads=4, fast_kv_heads=2, fast_head_dim=64, fast_ffn=768,
                       num_codebooks=4, codebook_size=1024, context_length=4096,
                       linear_type=linear_type, seed=seed)


def tiny_codec(seed: int = 0) -> ModelConfig:
    """A tiny Dual-AR whose codes the s2-pro codec decodes: 2 Slow-AR layers
    (d 512), 4096 text + 4096 semantic ids, 1 Fast-AR layer, 10 codebooks x
    1024 (the codec's residual codebook size).  For end-to-end pipeline tests."""
    return ModelConfig(name="tinycodec", slow_layers=2, d=512, heads=8, kv_heads=2, head_dim=64,
                       ffn=1536, vocab=8192, sem_begin=4096, sem_end=8191, fast_layers=1,
                       fast_heads=4, fast_kv_heads=2, fast_head_dim=64, fast_ffn=768,
                       num_codebooks=10, codebook_size=1024, context_length=4096, seed=seed)


def s2pro(seed: int = 1, linear_type: int = GGML_F16, slow_layers: int = 36,
          fast_layers: int = 4) -> ModelConfig:
    """C2..C5 shapes: 36 Slow-AR layers, d 2560, 32/8 heads x 128, FFN 9728,
    vocab 155,776 (semantic 151,678..155,773); Fast-AR 4 layers of the same
    layer shape; 10 codebooks x 4096.  `slow_layers`/`fast_layers` only shrink
    the stack for quick parity cases; the benchmark uses the full stack."""
    return ModelConfig(name="s2pro", slow_layers=slow_layers, d=2560, heads=32, kv_heads=8,
                       head_dim=128, ffn=9728, vocab=155776, sem_begin=151678, sem_end=155773,
                       fast_layers=fast_layers, fast_heads=32, fast_kv_heads=8, fast_head_dim=128,
                       fast_ffn=9728, num_codebooks=10, codebook_size=4096,
                       context_length=32768, linear_type=linear_type, seed=seed)


# <|im_end|> of the Qwen-style tokenizer the reference uses (a text id).
S2PRO_IM_END = 151645
TINY_IM_END = 4000

C1 = Workload(tiny(seed=0), prompt_len=64, frames=32, prompt_seed=0, im_end_id=TINY_IM_END)
C2 = Workload(s2pro(seed=1), prompt_len=512, frames=256, prompt_seed=1, im_end_id=S2PRO_IM_END)
C3 = Workload(s2pro(seed=2, linear_type=GGML_Q8_0), prompt_len=512, frames=256, prompt_seed=2,
              im_end_id=S2PRO_IM_END)
C4 = Workload(s2pro(seed=3), prompt_len=1024, frames=512, prompt_seed=3, im_end_id=S2PRO_IM_END,
              batch=64, prompt_len_min=128)
C5 = Workload(s2pro(seed=4, linear_type=GGML_Q4_K), prompt_len=8192, frames=256, prompt_seed=4,
              im_end_id=S2PRO_IM_END)

WORKLOADS = {"C1": C1, "C2": C2, "C3": C3, "C4": C4, "C5": C5}

# Profiling case: C2's layer shapes with 4 Slow-AR and 1 Fast-AR layers (about
# 2 GB on the device), small enough for full ncu captures of C2's kernels.
C2S = Workload(s2pro(seed=1, slow_layers=4, fast_layers=1), prompt_len=64, frames=4,
               prompt_seed=1, im_end_id=S2PRO_IM_END)
# Profiling case of the batched step: C4's shapes and batch with 4 Slow-AR and
# 1 Fast-AR layers (about 3 GB on the device with the 64 caches).
C4S = Workload(s2pro(seed=3, slow_layers=4, fast_layers=1), prompt_len=1024, frames=4, prompt_seed=3,
               im_end_id=S2PRO_IM_END, batch=64, prompt_len_min=128)
PROFILING = {"C2S": C2S, "C4S": C4S}


def weight_bytes_per_frame(m: ModelConfig) -> dict:
    """Algorithmic HBM bytes of one batch-1 frame, excluding the KV term:
    every Slow-AR layer once, the masked LM head (semantic rows + im_end),
    and K-1 Fast-AR passes over the Fast-AR layers and fast_output."""
    bw = {GGML_F16: 2.0, GGML_Q8_0: 34 / 32, GGML_Q4_K: 144 / 256}[m.linear_type]
    qs, kvs = m.heads * m.head_dim, m.kv_heads * m.head_dim
    slow_layer = m.d * (qs + 2 * kvs) + qs * m.d + 3 * m.d * m.ffn
    fqs, fkvs = m.fast_heads * m.fast_head_dim, m.fast_kv_heads * m.fast_head_dim
    fast_layer = m.d * (fqs + 2 * fkvs) + fqs * m.d + 3 * m.d * m.fast_ffn
    n_sem = m.sem_end - m.sem_begin + 1 + 1
    passes = m.num_codebooks - 1
    return {
        "slow": m.slow_layers * slow_layer * bw,
        "lm_head": n_sem * m.d * 2.0,
        "fast": passes * (m.fast_layers * fast_layer + m.d * m.codebook_size) * bw,
        "embed_rows": (1 + m.num_codebooks + passes) * m.d * 2.0,
    }


def kv_bytes_per_position(m: ModelConfig) -> int:
    """f16 K and V of one attended position over all Slow-AR layers."""
    return m.slow_layers * 2 * m.kv_heads * m.head_dim * 2
