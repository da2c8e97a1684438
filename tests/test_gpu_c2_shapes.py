"""Parity at the benchmark's layer shapes: C2's dimensions (d 2560, 32/8
heads of 128, FFN 9728, vocab 155,776, 10 codebooks x 4096) with 2 Slow-AR
layers and 1 Fast-AR layer, against the CPU oracle.

Covers what the C1-shaped tests cannot:
- head_dim 128 in every attention kernel (the prompt-chunk attention, the
  engine's attention ops, the batched rows attention);
- the engine's ring tiles at d 2560 / FFN 9728;
- the masked LM head over the 4,096 semantic rows of a 155,776 vocabulary.

Criteria as in the other parity tests: logits within 2e-2 relative
(max|a-b| / max|b|) on the allowed ids; greedy ids equal to the oracle's
wherever its top-2 margin exceeds 2e-2 x max|logit|.
"""
import numpy as np
import pytest

from fish_s2pro_b200 import configs
from oracle import oracle as o

pytestmark = pytest.mark.gpu

TOL = 2e-2
M = configs.s2pro(seed=5, slow_layers=2, fast_layers=1)
IM_END = configs.S2PRO_IM_END


def rel_err(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    fin = np.isfinite(b)
    assert np.array_equal(fin, np.isfinite(a))
    return float(np.max(np.abs(a[fin] - b[fin])) / np.max(np.abs(b[fin])))


def greedy_consistent(choice, ref_logits):
    lg = np.asarray(ref_logits, np.float64)
    fin = np.isfinite(lg)
    order = np.argsort(-np.where(fin, lg, -np.inf), kind="stable")
    if choice == order[0]:
        return True
    return lg[order[0]] - lg[choice] <= TOL * np.max(np.abs(lg[fin]))


def prompt(n, seed):
    rng = np.random.default_rng(seed)
    p = np.zeros((M.num_codebooks + 1, n), dtype=np.uint32)
    p[0] = rng.integers(0, M.sem_begin, size=n, dtype=np.uint32)
    return p


@pytest.fixture(scope="module")
def path(model_dir):
    from fish_s2pro_b200 import synth
    return synth.cached_gguf(M, model_dir)


@pytest.fixture(scope="module")
def cpu(path):
    om = o.OracleModel(str(path), max_seq_len=96, mode=0)
    yield om
    om.close()


@pytest.fixture(scope="module")
def gpu(path):
    from fish_s2pro_b200 import SlowArState
    st = SlowArState.open(path, max_seq_len=96, max_batch=2)
    yield st
    st.close()


def test_prefill_and_steps_match_oracle(gpu, cpu):
    """A 40-token prompt (the prompt-chunk path with its tiled attention),
    then two teacher-forced steps (per-op kernels)."""
    flat = prompt(40, 1).T.reshape(-1).astype(np.int32)
    gpu.reset()
    cpu.reset()
    g = gpu.prefill(flat, logits="allowed", im_end_id=IM_END)
    h, lg = cpu.eval(flat, allowed_only=True, im_end_id=IM_END)
    assert rel_err(g.logits, lg) < TOL
    assert rel_err(g.hidden, h) < TOL
    sem = slice(M.sem_begin, M.sem_end + 1)
    for _ in range(2):
        main = M.sem_begin + int(np.argmax(lg[sem]))
        codes = [main - M.sem_begin] + [int(c) for c in (np.arange(1, M.num_codebooks) * 37) % M.codebook_size]
        step = [main] + codes
        g = gpu.step(step, logits="allowed", im_end_id=IM_END)
        h, lg = cpu.eval(step, allowed_only=True, im_end_id=IM_END)
        assert rel_err(g.logits, lg) < TOL
        assert rel_err(g.hidden, h) < TOL


def replay(cpu, p, codes):
    """The oracle's greedy choices along the GPU's trajectory (margin rule)."""
    cpu.reset()
    h, lg = cpu.eval(p.T.reshape(-1).astype(np.int32), allowed_only=True, im_end_id=IM_END)
    for f in range(codes.shape[1]):
        assert greedy_consistent(int(codes[0, f]), lg[M.sem_begin:M.sem_end + 1]), f
        for k in range(1, M.num_codebooks):
            assert greedy_consistent(int(codes[k, f]), cpu.fast_prefix_logits(h, codes[:k, f].tolist())), (f, k)
        h, lg = cpu.eval([M.sem_begin + int(codes[0, f])] + codes[:, f].tolist(), allowed_only=True,
                         im_end_id=IM_END)


def test_engine_generation_matches_oracle(gpu, cpu):
    from fish_s2pro_b200 import FastArWeights, GenerateParams, PromptTensor, SeededRng, generate_codes
    p = prompt(20, 2)
    frames = 4
    res = generate_codes(gpu, IM_END, gpu.graph_spec(), PromptTensor(p.shape[0], p.shape[1], p.reshape(-1)),
                         GenerateParams(frames, 0.0, 1.0, 0, 2 * frames + 2), FastArWeights.from_state(gpu),
                         SeededRng(0))
    assert res.n_frames == frames
    replay(cpu, p, res.codes.reshape(M.num_codebooks, frames))


def test_batched_generation_matches_oracle(gpu, cpu):
    from fish_s2pro_b200 import FastArWeights, GenerateParams, PromptTensor, SeededRng, generate_codes_batch
    ps = [prompt(18, 3), prompt(9, 4)]
    frames = 3
    res = generate_codes_batch(gpu, IM_END, gpu.graph_spec(),
                               [PromptTensor(p.shape[0], p.shape[1], p.reshape(-1)) for p in ps],
                               GenerateParams(frames, 0.0, 1.0, 0, 2 * frames + 2), FastArWeights.from_state(gpu),
                               [SeededRng(0), SeededRng(1)])
    for p, r in zip(ps, res):
        assert r.n_frames == frames
        replay(cpu, p, r.codes.reshape(M.num_codebooks, frames))
