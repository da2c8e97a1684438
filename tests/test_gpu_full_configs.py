"""Parity at the configurations the benchmark times, against the CPU oracle.

Models:
- C2: the full 36-layer f16 S2-Pro-shaped model of BASELINE configs[1]
  (the very file bench.py decodes);
- C3 / C5: the full 36-layer Q8_0 / Q4_K models of configs[2] / configs[4];
- C3S / C5S: Q8_0 / Q4_K at the same layer shapes with 2 Slow-AR and 1
  Fast-AR layers, for the cases that are too slow on the CPU at 36 layers.

What runs where:
- the prompt goes through the rows path (prompt-chunk GEMMs and attention;
  quantized models through the per-layer f16 dequantisation);
- teacher-forced steps go through s2d_step, which runs the persistent
  engine's Slow-AR step program (the quantized models on the engine's Q8_0 /
  Q4_K ring slots: 1,024-column K-slices, Q4_K's 38-superblock w2);
- Fast-AR codebook logits through forward_codebook_prefix and codebook
  choices through generate_codebooks_for_semantic (per-op kernels and the
  device sampler);
- free-running greedy generation through generate_codes (the frame graph:
  the engine's Fast-AR pass programs and Slow-AR step program), replayed
  teacher-forced on the oracle.

Criteria: logits within 2e-2 relative error
(max|a-b| / max|b| over the allowed ids) for f16, 5e-2 for Q8_0 / Q4_K;
greedy ids equal to the oracle's wherever its top-2 margin exceeds that
tolerance times max|logit|; dequantised weights bit-exact.  Quantized
parity is pinned to the oracle's restatement of ggml's published block
formats only: the reference is F16-only (registry.rs:332-339).
Reference loops: slow_ar.rs:1161-1213 (decode layers), fast_ar.rs:360-437
(codebook prefix), generate.rs:117-221 (generate_codes).
"""
import numpy as np
import pytest

from fish_s2pro_b200 import configs
from oracle import oracle as o

pytestmark = pytest.mark.gpu

Q8, Q4 = configs.GGML_Q8_0, configs.GGML_Q4_K
MODELS = {
    "C2": (configs.C2.model, 2e-2),
    "C3": (configs.C3.model, 5e-2),
    "C5": (configs.C5.model, 5e-2),
    "C3S": (configs.s2pro(seed=6, linear_type=Q8, slow_layers=2, fast_layers=1), 5e-2),
    "C5S": (configs.s2pro(seed=7, linear_type=Q4, slow_layers=2, fast_layers=1), 5e-2),
}
IM_END = configs.S2PRO_IM_END
MAX_SEQ = 64


def rel_err(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    fin = np.isfinite(b)
    assert np.array_equal(fin, np.isfinite(a))
    return float(np.max(np.abs(a[fin] - b[fin])) / np.max(np.abs(b[fin])))


def greedy_consistent(choice, ref_logits, tol):
    lg = np.asarray(ref_logits, np.float64)
    fin = np.isfinite(lg)
    best = int(np.argmax(np.where(fin, lg, -np.inf)))
    if choice == best:
        return True
    return lg[best] - lg[choice] <= tol * np.max(np.abs(lg[fin]))


def prompt(m, n, seed):
    rng = np.random.default_rng(seed)
    p = np.zeros((m.num_codebooks + 1, n), dtype=np.uint32)
    p[0] = rng.integers(0, m.sem_begin, size=n, dtype=np.uint32)
    return p


class Pair:
    """The GPU handle and the oracle on one model file."""

    def __init__(self, key, model_dir):
        from fish_s2pro_b200 import SlowArState, synth
        self.m, self.tol = MODELS[key]
        self.path = synth.cached_gguf(self.m, model_dir)
        # the layer-shape variants also decode batches of 2 sequences
        self.gpu = SlowArState.open(self.path, max_seq_len=MAX_SEQ, max_batch=2 if key.endswith("S") else 1)
        self.cpu = o.OracleModel(str(self.path), max_seq_len=MAX_SEQ, mode=0)

    def close(self):
        self.gpu.close()
        self.cpu.close()


_open = {}


@pytest.fixture(scope="module")
def pairs(model_dir):
    def get(key):
        if key not in _open:
            # one model resident at a time keeps host and device memory bounded
            for k in list(_open):
                _open.pop(k).close()
            _open[key] = Pair(key, model_dir)
        return _open[key]
    yield get
    for k in list(_open):
        _open.pop(k).close()


def _prefill(p, n=12, seed=11):
    flat = prompt(p.m, n, seed).T.reshape(-1).astype(np.int32)
    p.gpu.reset()
    p.cpu.reset()
    g = p.gpu.prefill(flat, logits="allowed", im_end_id=IM_END)
    h, lg = p.cpu.eval(flat, allowed_only=True, im_end_id=IM_END)
    return g, h, lg


def check_steps(p, key):
    """A 12-token prompt on the rows path, then two teacher-forced steps on
    the engine's step program: allowed logits and post-norm hidden."""
    m = p.m
    g, h, lg = _prefill(p)
    assert rel_err(g.logits, lg) < p.tol, key
    assert rel_err(g.hidden, h) < p.tol, key
    sem = slice(m.sem_begin, m.sem_end + 1)
    assert greedy_consistent(int(np.argmax(g.logits[sem])), lg[sem], p.tol)
    for i in range(2):
        main = m.sem_begin + int(np.argmax(lg[sem]))
        codes = [main - m.sem_begin] + [int(c) for c in (np.arange(1, m.num_codebooks) * (37 + i)) %
                                        m.codebook_size]
        step = [main] + codes
        g = p.gpu.step(step, logits="allowed", im_end_id=IM_END)
        h, lg = p.cpu.eval(step, allowed_only=True, im_end_id=IM_END)
        assert rel_err(g.logits, lg) < p.tol, (key, i)
        assert rel_err(g.hidden, h) < p.tol, (key, i)
        assert greedy_consistent(int(np.argmax(g.logits[sem])), lg[sem], p.tol), (key, i)
    assert p.gpu.n_past() == 14


def check_fast(p, key):
    """One frame's Fast-AR codebook logits and greedy codebook choices on the
    oracle's slow hidden."""
    from fish_s2pro_b200 import (FastArWeights, SamplerParams, SeededRng, forward_codebook_prefix,
                                 generate_codebooks_for_semantic)
    m = p.m
    _, h, lg = _prefill(p, n=9, seed=12)
    sem_code = int(np.argmax(lg[m.sem_begin:m.sem_end + 1]))
    spec = p.gpu.graph_spec()
    fw = FastArWeights.from_state(p.gpu)
    got = generate_codebooks_for_semantic(h, sem_code, spec, fw, SamplerParams(0.0, 1.0, 0), SeededRng(0))
    assert got[0] == sem_code
    for k in range(1, m.num_codebooks):
        cl = p.cpu.fast_prefix_logits(h, got[:k])
        gl = forward_codebook_prefix(h, got[:k], spec, fw)
        assert rel_err(gl, cl) < p.tol, (key, k)
        assert greedy_consistent(int(got[k]), cl, p.tol), (key, k)


def check_generation(p, key, frames=4):
    """Free-running greedy frames on the frame graph, replayed on the oracle:
    every semantic and codebook choice obeys the margin rule."""
    from fish_s2pro_b200 import FastArWeights, GenerateParams, PromptTensor, SeededRng, generate_codes
    m = p.m
    pr = prompt(m, 10, 13)
    res = generate_codes(p.gpu, IM_END, p.gpu.graph_spec(),
                         PromptTensor(pr.shape[0], pr.shape[1], pr.reshape(-1)),
                         GenerateParams(frames, 0.0, 1.0, 0, 2 * frames + 2), FastArWeights.from_state(p.gpu),
                         SeededRng(0))
    assert res.n_frames == frames
    codes = res.codes.reshape(m.num_codebooks, frames)
    p.cpu.reset()
    h, lg = p.cpu.eval(pr.T.reshape(-1).astype(np.int32), allowed_only=True, im_end_id=IM_END)
    for f in range(frames):
        assert greedy_consistent(int(codes[0, f]), lg[m.sem_begin:m.sem_end + 1], p.tol), (key, f)
        for k in range(1, m.num_codebooks):
            cl = p.cpu.fast_prefix_logits(h, codes[:k, f].tolist())
            assert greedy_consistent(int(codes[k, f]), cl, p.tol), (key, f, k)
        h, lg = p.cpu.eval([m.sem_begin + int(codes[0, f])] + codes[:, f].tolist(), allowed_only=True,
                           im_end_id=IM_END)


def check_dequant(p, key):
    """Dequantised weights at d 2560 / FFN 9728: WQKV (10 Q4_K superblocks or
    80 Q8_0 blocks per row), w2 (38 superblocks / 304 blocks per row) and the
    Fast-AR output head."""
    g = o.Gguf(p.path)
    names = ("layers.1.attention.wqkv.weight", "layers.1.feed_forward.w2.weight", "fast_output.weight",
             "fast_layers.0.feed_forward.w1.weight")
    seen = 0
    for t in g.tensors():
        if t["name"] in names:
            n = int(np.prod(t["dims"]))
            got = p.gpu.dequant_tensor(t["name"], n)
            want = o.dequant(t["type"], g.tensor_bytes(t["name"]), n)
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), t["name"]
            seen += 1
    assert seen == len(names)


def _replay(p, key, pr, codes):
    """The oracle's greedy choices along a GPU trajectory (margin rule)."""
    m = p.m
    p.cpu.reset()
    h, lg = p.cpu.eval(pr.T.reshape(-1).astype(np.int32), allowed_only=True, im_end_id=IM_END)
    for f in range(codes.shape[1]):
        assert greedy_consistent(int(codes[0, f]), lg[m.sem_begin:m.sem_end + 1], p.tol), (key, f)
        for k in range(1, m.num_codebooks):
            cl = p.cpu.fast_prefix_logits(h, codes[:k, f].tolist())
            assert greedy_consistent(int(codes[k, f]), cl, p.tol), (key, f, k)
        h, lg = p.cpu.eval([m.sem_begin + int(codes[0, f])] + codes[:, f].tolist(), allowed_only=True,
                           im_end_id=IM_END)


def check_batch(p, key, frames=3):
    """Batched greedy generation of two sequences (the rows path's GEMMs over
    the resident f16 expansion of the quantized linears), each replayed on
    the oracle."""
    from fish_s2pro_b200 import (FastArWeights, GenerateParams, PromptTensor, SeededRng,
                                 generate_codes_batch)
    m = p.m
    prs = [prompt(m, 11, 21), prompt(m, 8, 22)]
    res = generate_codes_batch(p.gpu, IM_END, p.gpu.graph_spec(),
                               [PromptTensor(x.shape[0], x.shape[1], x.reshape(-1)) for x in prs],
                               GenerateParams(frames, 0.0, 1.0, 0, 2 * frames + 2), FastArWeights.from_state(p.gpu),
                               [SeededRng(0), SeededRng(1)])
    for pr, r in zip(prs, res):
        assert r.n_frames == frames
        _replay(p, key, pr, r.codes.reshape(m.num_codebooks, frames))


CHECKS = {"steps": check_steps, "fast": check_fast, "generation": check_generation, "dequant": check_dequant,
          "batch": check_batch}


# one test function per model, so that each model file is uploaded once


@pytest.mark.parametrize("check", ["steps", "fast", "generation"])
def test_c2_full_depth(pairs, check):
    CHECKS[check](pairs("C2"), "C2")


@pytest.mark.parametrize("check", ["steps"])
def test_c3_full_depth(pairs, check):
    CHECKS[check](pairs("C3"), "C3")


@pytest.mark.parametrize("check", ["steps"])
def test_c5_full_depth(pairs, check):
    CHECKS[check](pairs("C5"), "C5")


@pytest.mark.parametrize("check", ["steps", "fast", "generation", "dequant", "batch"])
def test_c3_layer_shapes(pairs, check):
    CHECKS[check](pairs("C3S"), "C3S")


@pytest.mark.parametrize("check", ["steps", "fast", "generation", "dequant", "batch"])
def test_c5_layer_shapes(pairs, check):
    CHECKS[check](pairs("C5S"), "C5S")
