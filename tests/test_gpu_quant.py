"""Parity of the sm_100a path on quantized linears (Q8_0 for C3, Q4_K for C5)
against the CPU oracle, on C1-shaped models.

Criteria: dequantised weights bit-exact; logits within
5e-2 relative error (max|a-b| / max|b|) for quantized weights; greedy ids
equal to the oracle's wherever its top-2 margin exceeds that tolerance times
max|logit|.  The persistent engine (decode frames), the batched prefill and
the per-op kernels (single steps, Fast-AR prefix API) all run here.
"""
import numpy as np
import pytest

from fish_s2pro_b200 import configs
from oracle import oracle as o

pytestmark = pytest.mark.gpu

TOL = 5e-2
TYPES = {"q8_0": configs.GGML_Q8_0, "q4_k": configs.GGML_Q4_K}


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


@pytest.fixture(scope="module", params=sorted(TYPES))
def quant(request, model_dir):
    from fish_s2pro_b200 import SlowArState, synth
    m = configs.tiny(seed=7, linear_type=TYPES[request.param])
    path = synth.cached_gguf(m, model_dir)
    st = SlowArState.open(path, max_seq_len=256)
    cpu = o.OracleModel(path, max_seq_len=256, mode=0)
    yield m, path, st, cpu
    st.close()
    cpu.close()


def test_dequant_is_bit_exact(quant):
    m, path, st, _ = quant
    g = o.Gguf(path)
    names = ("layers.0.attention.wqkv.weight", "layers.1.feed_forward.w2.weight",
             "fast_layers.0.feed_forward.w1.weight", "fast_output.weight")
    for t in g.tensors():
        if t["name"] in names:
            assert t["type"] == m.linear_type, t["name"]
            n = int(np.prod(t["dims"]))
            got = st.dequant_tensor(t["name"], n)
            want = o.dequant(t["type"], g.tensor_bytes(t["name"]), n)
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), t["name"]


def test_prefill_and_teacher_forced_steps(quant):
    """Batched prefill, then Slow-AR single steps and Fast-AR prefix logits on
    the oracle's greedy choices."""
    m, _, st, cpu = quant
    from fish_s2pro_b200 import FastArWeights, forward_codebook_prefix
    wl = configs.C1
    flat = wl.prompt().T.reshape(-1).astype(np.int32)
    st.reset()
    cpu.reset()
    g = st.prefill(flat, logits="full")
    h, lg = cpu.eval(flat)
    assert rel_err(g.logits, lg) < TOL
    assert rel_err(g.hidden, h) < TOL
    fw = FastArWeights.from_state(st)
    spec = st.graph_spec()
    sem = slice(m.sem_begin, m.sem_end + 1)
    for f in range(3):
        main = m.sem_begin + int(np.argmax(lg[sem]))
        codes = [main - m.sem_begin]
        for k in range(1, m.num_codebooks):
            gl = forward_codebook_prefix(h, codes, spec, fw)
            cl = cpu.fast_prefix_logits(h, codes)
            assert rel_err(gl, cl) < TOL, (f, k)
            codes.append(int(np.argmax(cl)))
        step = [main] + codes
        g = st.step(step, logits="full")
        h, lg = cpu.eval(step)
        assert rel_err(g.logits, lg) < TOL, f
        assert rel_err(g.hidden, h) < TOL, f


def test_generate_codes_greedy(quant):
    """Free-running greedy generation through the persistent engine: every
    choice is the oracle's greedy choice on the GPU's trajectory, up to the
    margin rule."""
    m, _, st, cpu = quant
    from fish_s2pro_b200 import (FastArWeights, GenerateParams, PromptTensor, SeededRng,
                                 generate_codes)
    wl = configs.C1
    gp = wl.gen_params(greedy=True)
    frames = 8
    prompt = wl.prompt()
    res = generate_codes(st, gp["im_end_id"], st.graph_spec(),
                         PromptTensor(prompt.shape[0], prompt.shape[1], prompt.reshape(-1)),
                         GenerateParams(frames, gp["temperature"], gp["top_p"], gp["top_k"],
                                        2 * frames + 2),
                         FastArWeights.from_state(st), SeededRng(0))
    assert res.n_frames == frames
    codes = res.codes.reshape(m.num_codebooks, res.n_frames)
    cpu.reset()
    flat = prompt.T.reshape(-1).astype(np.int32)
    h, lg = cpu.eval(flat, allowed_only=True, im_end_id=gp["im_end_id"])
    for f in range(res.n_frames):
        assert greedy_consistent(int(codes[0, f]), lg[m.sem_begin:m.sem_end + 1]), f
        for k in range(1, m.num_codebooks):
            cl = cpu.fast_prefix_logits(h, codes[:k, f].tolist())
            assert greedy_consistent(int(codes[k, f]), cl), (f, k)
        main = m.sem_begin + int(codes[0, f])
        h, lg = cpu.eval([main] + codes[:, f].tolist(), allowed_only=True, im_end_id=gp["im_end_id"])
