"""Long prompts on C1-shaped models against the CPU oracle: a 1,200-token
prompt is prefilled in three chunks of up to 512 rows (the prompt-chunk
attention reaching back over earlier chunks), then decoded by the engine
at positions past 1,200 (its attention split over many position ranges),
for f16 and Q4_K weights.  Criteria as in the other parity tests."""
import numpy as np
import pytest

from fish_s2pro_b200 import configs
from oracle import oracle as o

pytestmark = pytest.mark.gpu

N_PROMPT = 1200


def rel_err(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    fin = np.isfinite(b)
    assert np.array_equal(fin, np.isfinite(a))
    return float(np.max(np.abs(a[fin] - b[fin])) / np.max(np.abs(b[fin])))


def greedy_consistent(choice, ref_logits, tol):
    lg = np.asarray(ref_logits, np.float64)
    fin = np.isfinite(lg)
    order = np.argsort(-np.where(fin, lg, -np.inf), kind="stable")
    if choice == order[0]:
        return True
    return lg[order[0]] - lg[choice] <= tol * np.max(np.abs(lg[fin]))


@pytest.mark.parametrize("lt", [configs.GGML_F16, configs.GGML_Q4_K])
def test_long_prompt_prefill_and_decode(lt, model_dir):
    from fish_s2pro_b200 import (FastArWeights, GenerateParams, PromptTensor, SeededRng, SlowArState,
                                 generate_codes, synth)
    m = configs.tiny(seed=11, linear_type=lt)
    tol = 2e-2 if lt == configs.GGML_F16 else 5e-2
    path = synth.cached_gguf(m, model_dir)
    rng = np.random.default_rng(21)
    p = np.zeros((m.num_codebooks + 1, N_PROMPT), dtype=np.uint32)
    p[0] = rng.integers(0, m.sem_begin, size=N_PROMPT, dtype=np.uint32)
    flat = p.T.reshape(-1).astype(np.int32)
    im_end = configs.TINY_IM_END
    st = SlowArState.open(path, max_seq_len=N_PROMPT + 32)
    cpu = o.OracleModel(str(path), max_seq_len=N_PROMPT + 32, mode=0)
    try:
        g = st.prefill(flat, logits="full")
        h, lg = cpu.eval(flat)
        assert rel_err(g.logits, lg) < tol
        assert rel_err(g.hidden, h) < tol
        frames = 6
        res = generate_codes(st, im_end, st.graph_spec(), PromptTensor(p.shape[0], p.shape[1], p.reshape(-1)),
                             GenerateParams(frames, 0.0, 1.0, 0, 2 * frames + 2), FastArWeights.from_state(st),
                             SeededRng(0))
        assert res.n_frames == frames
        codes = res.codes.reshape(m.num_codebooks, frames)
        cpu.reset()
        h, lg = cpu.eval(flat, allowed_only=True, im_end_id=im_end)
        for f in range(frames):
            assert greedy_consistent(int(codes[0, f]), lg[m.sem_begin:m.sem_end + 1], tol), f
            for k in range(1, m.num_codebooks):
                assert greedy_consistent(int(codes[k, f]), cpu.fast_prefix_logits(h, codes[:k, f].tolist()), tol)
            h, lg = cpu.eval([m.sem_begin + int(codes[0, f])] + codes[:, f].tolist(), allowed_only=True,
                             im_end_id=im_end)
    finally:
        st.close()
        cpu.close()
