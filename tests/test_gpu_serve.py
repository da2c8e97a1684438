"""Continuous batching (s2d_serve_* and fish_s2pro_b200.serve.TtsScheduler).

Requests join the batched frame between frames, in free slots, when the KV
pool has the pages their prompt and max_new_tokens need, and leave when they
finish.  Each row of the batched frame is computed on its own, so with the
reference's SeededRng a request's codes and final RNG state must not depend
on its slot, its neighbours or when it joined: the interleaved run must equal
running every request alone through the same session, bit for bit.  Greedy
requests are also replayed on the CPU oracle under the margin rule
(logits tolerance 2e-2 of max|logit|).
"""
import numpy as np
import pytest

from fish_s2pro_b200 import configs
from oracle import oracle as o

pytestmark = pytest.mark.gpu

TOL = 2e-2
M = configs.C1.model
FRAMES = 10


def greedy_consistent(choice, ref_logits):
    lg = np.asarray(ref_logits, np.float64)
    fin = np.isfinite(lg)
    order = np.argsort(-np.where(fin, lg, -np.inf), kind="stable")
    if choice == order[0]:
        return True
    return lg[order[0]] - lg[choice] <= TOL * np.max(np.abs(lg[fin]))


def requests(n, seed, lo=12, hi=60):
    """n prompts of lo..hi columns (text ids in row 0, codebook rows 0)."""
    from fish_s2pro_b200 import PromptTensor
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        cols = int(rng.integers(lo, hi + 1))
        p = np.zeros((M.num_codebooks + 1, cols), dtype=np.uint32)
        p[0] = rng.integers(0, M.sem_begin, size=cols, dtype=np.uint32)
        out.append(PromptTensor(p.shape[0], cols, p.reshape(-1)))
    return out


def params(greedy):
    from fish_s2pro_b200 import GenerateParams
    if greedy:
        return GenerateParams(FRAMES, 0.0, 1.0, 0, 2 * FRAMES + 2)
    return GenerateParams(FRAMES, 0.8, 0.9, 30, 2 * FRAMES + 2)


@pytest.fixture(scope="module")
def gpu(tiny_gguf):
    from fish_s2pro_b200 import SlowArState
    # 4 slots; 6 pages of 64 positions: at most 3 requests of <= 72 positions at once
    st = SlowArState.open(tiny_gguf, max_seq_len=128, max_batch=4, kv_pages=6)
    yield st
    st.close()


@pytest.mark.parametrize("greedy", [False, True], ids=["sampled", "greedy"])
def test_interleaved_serving_equals_requests_alone(gpu, greedy):
    from fish_s2pro_b200 import SeededRng, TtsScheduler
    reqs = requests(9, 7 if greedy else 8)
    seeds = [100 + i for i in range(len(reqs))]
    alone = {}
    for i, r in enumerate(reqs):
        sch = TtsScheduler(gpu, configs.C1.im_end_id, params(greedy), frames_per_step=2)
        rid = sch.submit(r, SeededRng(seeds[i]))
        alone[i] = sch.run()[rid]
    sch = TtsScheduler(gpu, configs.C1.im_end_id, params(greedy), frames_per_step=3)
    ids = [sch.submit(r, SeededRng(seeds[i])) for i, r in enumerate(reqs)]
    got = sch.run()
    assert sorted(got) == sorted(ids)
    joined = sorted({got[i].admitted_frame for i in ids})
    assert len(joined) >= 3 and joined[0] == 0  # requests joined a running batch
    for i, rid in enumerate(ids):
        a, b = alone[i], got[rid]
        assert b.result.n_frames == a.result.n_frames == FRAMES
        assert np.array_equal(b.result.codes, a.result.codes), i
        assert b.rng_state == a.rng_state, i


def test_serving_greedy_matches_oracle(gpu, tiny_gguf):
    from fish_s2pro_b200 import SeededRng, TtsScheduler
    reqs = requests(5, 3)
    sch = TtsScheduler(gpu, configs.C1.im_end_id, params(True), frames_per_step=4)
    ids = [sch.submit(r, SeededRng(0)) for r in reqs]
    got = sch.run()
    cpu = o.OracleModel(tiny_gguf, max_seq_len=128, mode=0)
    try:
        for r, rid in zip(reqs, ids):
            codes = got[rid].result.codes.reshape(M.num_codebooks, FRAMES)
            prompt = np.asarray(r.data, np.uint32).reshape(r.rows, r.cols)
            cpu.reset()
            h, lg = cpu.eval(prompt.T.reshape(-1).astype(np.int32), allowed_only=True,
                             im_end_id=configs.C1.im_end_id)
            for f in range(FRAMES):
                assert greedy_consistent(int(codes[0, f]), lg[M.sem_begin:M.sem_end + 1]), (rid, f)
                for k in range(1, M.num_codebooks):
                    assert greedy_consistent(int(codes[k, f]), cpu.fast_prefix_logits(h, codes[:k, f].tolist())), \
                        (rid, f, k)
                h, lg = cpu.eval([M.sem_begin + int(codes[0, f])] + codes[:, f].tolist(), allowed_only=True,
                                 im_end_id=configs.C1.im_end_id)
    finally:
        cpu.close()


def test_admission_is_limited_by_free_pages(gpu):
    from fish_s2pro_b200 import S2dError, SeededRng, ServeSession
    reqs = requests(4, 11, lo=55)  # 65..70 positions: 2 pages of 64 each
    s = ServeSession(gpu, configs.C1.im_end_id, params(True))
    assert s.free_pages() == 6
    for slot in range(3):
        assert s.admit(slot, reqs[slot], SeededRng(slot).state)
    assert s.free_pages() == 0
    assert not s.admit(3, reqs[3], 0)  # S2D_EFULL: the fourth slot is free, the pages are not
    with pytest.raises(S2dError):
        s.admit(0, reqs[3], 0)  # slot 0 is taken
    status, frames = s.step(FRAMES + 2)
    assert list(status) == [2, 2, 2, 0] and list(frames[:3]) == [FRAMES] * 3
    for slot in range(3):
        codes, n, _ = s.collect(slot)
        assert n == FRAMES and codes.size == M.num_codebooks * FRAMES
    assert s.free_pages() == 6
    assert s.admit(3, reqs[3], 0)
    with pytest.raises(S2dError):
        s.collect(3)  # still running


def test_batch_call_after_serving(gpu):
    """generate_codes_batch deals the pool out again after a session."""
    from fish_s2pro_b200 import SeededRng, generate_codes_batch, FastArWeights
    reqs = requests(3, 5)
    res = generate_codes_batch(gpu, configs.C1.im_end_id, gpu.graph_spec(), reqs, params(True),
                               FastArWeights.from_state(gpu), [SeededRng(0) for _ in reqs])
    assert [r.n_frames for r in res] == [FRAMES] * 3
