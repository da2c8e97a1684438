"""Batched generation (s2d_generate_codes_batch, the C4 path) against the
CPU oracle on C1-shaped models.

Every sequence of a batch must behave like its own generate_codes call:
greedy choices equal the oracle's on the sequence's own trajectory wherever
the oracle's top-2 margin exceeds 2e-2 x max|logit| (the north star's
f16 rule); with the reference's SeededRng the sampled codes equal the
oracle's golden sampled codes.  Prompts have different lengths (5 takes the
per-op prefill, the others the batched prefill), so rows attend over
different positions in their own KV caches.
"""
import json
from pathlib import Path

import numpy as np
import pytest

from fish_s2pro_b200 import configs
from oracle import oracle as o

pytestmark = pytest.mark.gpu

TOL = 2e-2
GOLDEN = json.loads((Path(__file__).parent / "golden" / "c1_oracle.json").read_text())
LENS = (64, 5, 33, 12)

# Philox4x32-10 known-answer vectors (Random123 kat_vectors: counter, key, output)
PHILOX_KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


def greedy_consistent(choice, ref_logits):
    lg = np.asarray(ref_logits, np.float64)
    fin = np.isfinite(lg)
    order = np.argsort(-np.where(fin, lg, -np.inf), kind="stable")
    if choice == order[0]:
        return True
    return lg[order[0]] - lg[choice] <= TOL * np.max(np.abs(lg[fin]))


def prompts():
    """C1's prompt first, then seeded text prompts of the other lengths."""
    m = configs.C1.model
    out = [configs.C1.prompt()]
    rng = np.random.default_rng(11)
    for n in LENS[1:]:
        p = np.zeros((m.num_codebooks + 1, n), dtype=np.uint32)
        p[0] = rng.integers(0, m.sem_begin, size=n, dtype=np.uint32)
        out.append(p)
    return out


@pytest.fixture(scope="module")
def gpu(tiny_gguf):
    from fish_s2pro_b200 import SlowArState
    st = SlowArState.open(tiny_gguf, max_seq_len=256, max_batch=len(LENS))
    yield st
    st.close()


@pytest.fixture(scope="module")
def cpu(tiny_gguf):
    return o.OracleModel(tiny_gguf, max_seq_len=256, mode=0)


def run_batch(gpu, ps, gp, rngs, **kw):
    from fish_s2pro_b200 import FastArWeights, GenerateParams, PromptTensor, generate_codes_batch
    return generate_codes_batch(
        gpu, gp["im_end_id"], gpu.graph_spec(),
        [PromptTensor(p.shape[0], p.shape[1], p.reshape(-1)) for p in ps],
        GenerateParams(gp["max_new_tokens"], gp["temperature"], gp["top_p"], gp["top_k"],
                       gp["min_tokens_before_end"]),
        FastArWeights.from_state(gpu), rngs, **kw)


def test_philox_matches_published_vectors():
    import ctypes
    from fish_s2pro_b200 import lib
    for ctr, key, want in PHILOX_KAT:
        c = (ctypes.c_uint32 * 4)(*ctr)
        k = (ctypes.c_uint32 * 2)(*key)
        out = (ctypes.c_uint32 * 4)()
        assert lib().s2d_philox4x32_10(c, k, out) == 0
        assert tuple(out) == want


def test_batch_greedy_matches_oracle(gpu, cpu):
    check_batch_greedy(gpu, cpu)


def test_batch_greedy_on_tcgen05_gemm_matches_oracle(tiny_gguf, cpu, monkeypatch):
    """The same run with the rows path's linears on the tcgen05 GEMM."""
    from fish_s2pro_b200 import SlowArState
    monkeypatch.setenv("S2D_TCGEMM", "1")
    st = SlowArState.open(tiny_gguf, max_seq_len=256, max_batch=len(LENS))
    try:
        check_batch_greedy(st, cpu)
    finally:
        st.close()


def check_batch_greedy(gpu, cpu):
    from fish_s2pro_b200 import SeededRng
    m = configs.C1.model
    frames = 12
    gp = dict(max_new_tokens=frames, temperature=0.0, top_p=1.0, top_k=0,
              min_tokens_before_end=2 * frames + 2, im_end_id=configs.C1.im_end_id)
    ps = prompts()
    res = run_batch(gpu, ps, gp, [SeededRng(i) for i in range(len(ps))])
    assert res[0].profile.frames == frames * len(ps)
    for i, (p, r) in enumerate(zip(ps, res)):
        assert r.n_frames == frames, i
        codes = r.codes.reshape(m.num_codebooks, r.n_frames)
        cpu.reset()
        h, lg = cpu.eval(p.T.reshape(-1).astype(np.int32), allowed_only=True,
                         im_end_id=gp["im_end_id"])
        for f in range(r.n_frames):
            assert greedy_consistent(int(codes[0, f]), lg[m.sem_begin:m.sem_end + 1]), (i, f)
            for k in range(1, m.num_codebooks):
                cl = cpu.fast_prefix_logits(h, codes[:k, f].tolist())
                assert greedy_consistent(int(codes[k, f]), cl), (i, f, k)
            main = m.sem_begin + int(codes[0, f])
            h, lg = cpu.eval([main] + codes[:, f].tolist(), allowed_only=True,
                             im_end_id=gp["im_end_id"])


def test_batch_sampled_seeded_rng_matches_golden(gpu):
    """Sequence 0 is C1's prompt with the golden run's sampler and seed: its
    codes equal the oracle's sampled codes; the other sequences run beside it
    with their own RNG states."""
    from fish_s2pro_b200 import SeededRng
    gp = dict(GOLDEN["sampled_params"])
    ps = prompts()
    rngs = [SeededRng(GOLDEN["sampled_seed"])] + [SeededRng(100 + i) for i in range(1, len(ps))]
    res = run_batch(gpu, ps, gp, rngs)
    codes = res[0].codes.reshape(configs.C1.model.num_codebooks, res[0].n_frames)
    assert codes.tolist() == GOLDEN["sampled_codes"]
    # one draw per sample call: the first semantic sample, then K per frame
    k = configs.C1.model.num_codebooks
    want = o.SeededRng(GOLDEN["sampled_seed"])
    for _ in range(1 + res[0].n_frames * k):
        want.next_unit()
    assert rngs[0].state == want.state.value


def test_batch_philox_is_deterministic_and_counts_draws(gpu):
    from fish_s2pro_b200 import RNG_PHILOX, SeededRng
    frames = 6
    gp = dict(max_new_tokens=frames, temperature=0.8, top_p=0.9, top_k=30,
              min_tokens_before_end=2 * frames + 2, im_end_id=configs.C1.im_end_id)
    ps = prompts()
    runs = []
    for key in (1234, 1234, 99):
        rngs = [SeededRng(0) for _ in ps]
        res = run_batch(gpu, ps, gp, rngs, rng_kind=RNG_PHILOX, philox_key=key)
        k = configs.C1.model.num_codebooks
        assert [r.state for r in rngs] == [1 + frames * k] * len(ps)
        runs.append([r.codes.tolist() for r in res])
    assert runs[0] == runs[1]
    assert runs[0] != runs[2]
    # the same prompt twice: each sequence draws from its own stream
    same = [ps[0], ps[0]]
    res = run_batch(gpu, same, gp, [SeededRng(0), SeededRng(0)], rng_kind=RNG_PHILOX, philox_key=5)
    assert res[0].codes.tolist() != res[1].codes.tolist()


def test_batch_rejects_bad_arguments(gpu, tiny_gguf, model_dir):
    from fish_s2pro_b200 import S2dError, SeededRng, SlowArState, synth
    gp = dict(max_new_tokens=4, temperature=0.0, top_p=1.0, top_k=0, min_tokens_before_end=0,
              im_end_id=configs.C1.im_end_id)
    ps = prompts() + prompts()[:1]
    with pytest.raises(S2dError):
        run_batch(gpu, ps, gp, [SeededRng(0) for _ in ps])  # more than max_batch
    gp2 = dict(gp, max_new_tokens=250)
    with pytest.raises(S2dError):
        run_batch(gpu, prompts(), gp2, [SeededRng(0) for _ in LENS])  # exceeds max_seq
    # a quantized model decodes in batches too (over the f16 expansion of its
    # linears; parity in tests/test_gpu_full_configs.py)
    q = synth.cached_gguf(configs.tiny(seed=7, linear_type=configs.GGML_Q8_0), model_dir)
    st = SlowArState.open(q, max_seq_len=128, max_batch=2)
    try:
        res = run_batch(st, prompts()[:2], dict(gp, min_tokens_before_end=10), [SeededRng(0), SeededRng(1)])
        assert [r.n_frames for r in res] == [4, 4]
    finally:
        st.close()
