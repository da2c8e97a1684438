"""The Fast-AR of a frame as one persistent engine launch.

generate_codebooks_for_semantic (fast_ar.rs:440-470) runs K-1 dependent
passes, each followed by sample_token (sampling.rs:121-241).  The engine
runs them as one program: every pass's layers and head, a sampler op on one
CTA that writes the code and the next pass's input row, and attention that
reads the earlier positions from the WQKV words of the passes that produced
them instead of a KV cache.  The arithmetic is the per-pass path's, so the
codes and the RNG state must equal those of S2D_FAST_FRAME=0 (one launch per
pass) exactly, greedy and sampled, at C1's shapes (head_dim 64, 1,024-entry
codebooks) and at C2's (head_dim 128, 4,096 entries, d 2560); the greedy
codes are also replayed on the CPU oracle under the margin rule.
"""
import numpy as np
import pytest

from fish_s2pro_b200 import configs
from oracle import oracle as o

pytestmark = pytest.mark.gpu

TOL = 2e-2
C2S = configs.s2pro(seed=5, slow_layers=2, fast_layers=1)


def greedy_consistent(choice, ref_logits):
    lg = np.asarray(ref_logits, np.float64)
    fin = np.isfinite(lg)
    order = np.argsort(-np.where(fin, lg, -np.inf), kind="stable")
    if choice == order[0]:
        return True
    return lg[order[0]] - lg[choice] <= TOL * np.max(np.abs(lg[fin]))


def run(path, prompt, im_end, frames, temperature, top_p, top_k, seed, fast_frame, monkeypatch):
    from fish_s2pro_b200 import (FastArWeights, GenerateParams, PromptTensor, SeededRng, SlowArState,
                                 generate_codes)
    monkeypatch.setenv("S2D_FAST_FRAME", "1" if fast_frame else "0")
    with SlowArState.open(path, max_seq_len=prompt.shape[1] + frames + 8) as st:
        rng = SeededRng(seed)
        res = generate_codes(st, im_end, st.graph_spec(),
                             PromptTensor(prompt.shape[0], prompt.shape[1], prompt.reshape(-1)),
                             GenerateParams(frames, temperature, top_p, top_k, 2 * frames + 2),
                             FastArWeights.from_state(st), rng)
        return res.codes.copy(), res.n_frames, rng.state, res.profile.kernels_per_frame


def c2s_prompt(n, seed):
    rng = np.random.default_rng(seed)
    p = np.zeros((C2S.num_codebooks + 1, n), dtype=np.uint32)
    p[0] = rng.integers(0, C2S.sem_begin, size=n, dtype=np.uint32)
    return p


CASES = [
    # (name, temperature, top_p, top_k, seed)
    ("greedy", 0.0, 1.0, 0, 0),
    ("sampled_topk", 0.8, 0.9, 30, 11),
    ("sampled_sort", 1.0, 0.95, 0, 12),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("shape", ["c1", "c2s"])
def test_frame_program_equals_per_pass_launches(shape, case, model_dir, tiny_gguf, monkeypatch):
    from fish_s2pro_b200 import synth
    _, temperature, top_p, top_k, seed = case
    if shape == "c1":
        path, prompt, im_end, frames = tiny_gguf, configs.C1.prompt(), configs.C1.im_end_id, 12
    else:
        path, prompt, im_end, frames = synth.cached_gguf(C2S, model_dir), c2s_prompt(24, 3), configs.S2PRO_IM_END, 6
    one = run(path, prompt, im_end, frames, temperature, top_p, top_k, seed, True, monkeypatch)
    per = run(path, prompt, im_end, frames, temperature, top_p, top_k, seed, False, monkeypatch)
    assert one[1] == per[1] == frames
    assert np.array_equal(one[0], per[0])
    assert one[2] == per[2]  # the same RNG draws: one per codebook and semantic step
    # fast_init + the frame's Fast-AR + embedding + Slow-AR step + its sampler
    assert one[3] == 5 and per[3] > one[3]


def test_frame_program_greedy_matches_oracle(model_dir, monkeypatch):
    from fish_s2pro_b200 import synth
    path = synth.cached_gguf(C2S, model_dir)
    p = c2s_prompt(20, 2)
    frames = 4
    codes, n, _, _ = run(path, p, configs.S2PRO_IM_END, frames, 0.0, 1.0, 0, 0, True, monkeypatch)
    assert n == frames
    codes = codes.reshape(C2S.num_codebooks, frames)
    cpu = o.OracleModel(str(path), max_seq_len=96, mode=0)
    try:
        h, lg = cpu.eval(p.T.reshape(-1).astype(np.int32), allowed_only=True, im_end_id=configs.S2PRO_IM_END)
        for f in range(frames):
            assert greedy_consistent(int(codes[0, f]), lg[C2S.sem_begin:C2S.sem_end + 1]), f
            for k in range(1, C2S.num_codebooks):
                assert greedy_consistent(int(codes[k, f]), cpu.fast_prefix_logits(h, codes[:k, f].tolist())), (f, k)
            h, lg = cpu.eval([C2S.sem_begin + int(codes[0, f])] + codes[:, f].tolist(), allowed_only=True,
                             im_end_id=configs.S2PRO_IM_END)
    finally:
        cpu.close()
