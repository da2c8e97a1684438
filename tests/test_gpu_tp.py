"""Slow-AR tensor parallelism on 2 GPUs (s2d_open_tp) against the CPU oracle.

Two processes, one per GPU, open the same C1-shaped model as the ranks of
a 2-way tensor-parallel Slow-AR.  Both must return the same results; the
prefill and teacher-forced steps match the oracle's logits within the f16
(2e-2) or quantized (5e-2) tolerance; greedy generation (per-op frame graph
with the NCCL allreduces captured in it) follows the oracle up to the
margin rule, and the batched path agrees across ranks.  Skipped with fewer
than 2 GPUs.
"""
import numpy as np
import pytest

from fish_s2pro_b200 import configs
from oracle import oracle as o

pytestmark = pytest.mark.gpu

TP = 2


def n_gpus():
    import torch
    return torch.cuda.device_count()


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


def _rank(rank, nid, path, steps, generate, q):
    import torch  # noqa: F401  (NCCL in this process is the framework's)
    from fish_s2pro_b200 import (FastArWeights, GenerateParams, PromptTensor, SeededRng, SlowArState,
                                 generate_codes, generate_codes_batch)
    try:
        st = SlowArState.open(path, max_seq_len=256, device=rank, max_batch=2, tp=(TP, rank, nid))
        out = {}
        wl = configs.C1
        flat = wl.prompt().T.reshape(-1).astype(np.int32)
        g = st.prefill(flat, logits="full")
        out["prefill"] = (g.hidden, g.logits)
        out["steps"] = [st.step(s, logits="full").logits for s in steps]
        if generate:
            gp = wl.gen_params(greedy=True)
            frames = 12
            prompt = wl.prompt()
            pt = PromptTensor(prompt.shape[0], prompt.shape[1], prompt.reshape(-1))
            params = GenerateParams(frames, gp["temperature"], gp["top_p"], gp["top_k"], 2 * frames + 2)
            res = generate_codes(st, gp["im_end_id"], st.graph_spec(), pt, params,
                                 FastArWeights.from_state(st), SeededRng(0))
            out["codes"] = res.codes.reshape(wl.model.num_codebooks, res.n_frames)
            short = np.zeros((prompt.shape[0], 9), dtype=np.uint32)
            short[0] = prompt[0, :9]
            pts = [pt, PromptTensor(short.shape[0], short.shape[1], short.reshape(-1))]
            bres = generate_codes_batch(st, gp["im_end_id"], st.graph_spec(), pts,
                                        GenerateParams(6, 0.8, 0.9, 30, 14),
                                        FastArWeights.from_state(st), [SeededRng(1), SeededRng(2)])
            out["batch"] = [r.codes for r in bres]
        st.close()
        q.put((rank, out, None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, repr(e)))


def run_ranks(path, steps, generate):
    import torch.multiprocessing as mp

    from fish_s2pro_b200 import nccl_unique_id
    nid = nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, nid, str(path), steps, generate, q)) for r in range(TP)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in procs:
            r, out, err = q.get(timeout=300)
            assert err is None, f"rank {r}: {err}"
            res[r] = out
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return res


def teacher_forced(cpu, m, n_steps):
    """The oracle's prefill and greedy teacher-forced steps on C1's prompt."""
    flat = configs.C1.prompt().T.reshape(-1).astype(np.int32)
    cpu.reset()
    h, lg = cpu.eval(flat)
    pre = (h, lg)
    steps, logits = [], []
    for _ in range(n_steps):
        main = m.sem_begin + int(np.argmax(lg[m.sem_begin:m.sem_end + 1]))
        codes = [main - m.sem_begin]
        for k in range(1, m.num_codebooks):
            codes.append(int(np.argmax(cpu.fast_prefix_logits(h, codes))))
        steps.append([main] + codes)
        h, lg = cpu.eval(steps[-1])
        logits.append(lg)
    return pre, steps, logits


@pytest.mark.skipif("n_gpus() < 2")
@pytest.mark.parametrize("lt", [configs.GGML_F16, configs.GGML_Q4_K])
def test_tp2_matches_oracle_and_ranks_agree(lt, model_dir):
    import torch  # noqa: F401
    from fish_s2pro_b200 import synth
    m = configs.C1.model if lt == configs.GGML_F16 else configs.tiny(seed=7, linear_type=lt)
    path = synth.cached_gguf(m, model_dir)
    tol = 2e-2 if lt == configs.GGML_F16 else 5e-2
    cpu = o.OracleModel(str(path), max_seq_len=256, mode=0)
    try:
        pre, steps, ref = teacher_forced(cpu, m, 3)
        res = run_ranks(path, steps, generate=lt == configs.GGML_F16)
        for r in range(TP):
            h, lg = res[r]["prefill"]
            assert rel_err(lg, pre[1]) < tol and rel_err(h, pre[0]) < tol, r
            for i, lg in enumerate(res[r]["steps"]):
                assert rel_err(lg, ref[i]) < tol, (r, i)
        # every rank holds the same residual stream after each allreduce
        assert np.array_equal(res[0]["prefill"][1], res[1]["prefill"][1])
        if lt != configs.GGML_F16:
            return
        codes = res[0]["codes"]
        assert np.array_equal(codes, res[1]["codes"])
        assert all(np.array_equal(a, b) for a, b in zip(res[0]["batch"], res[1]["batch"]))
        # greedy trajectory of the TP run follows the oracle (margin rule)
        cpu.reset()
        flat = configs.C1.prompt().T.reshape(-1).astype(np.int32)
        im_end = configs.C1.im_end_id
        h, lg = cpu.eval(flat, allowed_only=True, im_end_id=im_end)
        for f in range(codes.shape[1]):
            assert greedy_consistent(int(codes[0, f]), lg[m.sem_begin:m.sem_end + 1], tol), f
            for k in range(1, m.num_codebooks):
                assert greedy_consistent(int(codes[k, f]), cpu.fast_prefix_logits(h, codes[:k, f].tolist()),
                                         tol), (f, k)
            h, lg = cpu.eval([m.sem_begin + int(codes[0, f])] + codes[:, f].tolist(), allowed_only=True,
                             im_end_id=im_end)
    finally:
        cpu.close()


# ---------------------------------------------------------------------------
# the persistent engine with the NVLink exchange, C2 layer shapes, 2 / 4 / 8 ranks
# ---------------------------------------------------------------------------

C2S_MODEL = configs.s2pro(seed=5, slow_layers=2, fast_layers=1)
C5S_MODEL = configs.s2pro(seed=7, linear_type=configs.GGML_Q4_K, slow_layers=2, fast_layers=1)


def _engine_rank(rank, n, nid, path, prompt, steps, frames, q):
    import torch  # noqa: F401
    from fish_s2pro_b200 import (FastArWeights, GenerateParams, PromptTensor, SeededRng, SlowArState,
                                 generate_codes)
    try:
        im_end = configs.S2PRO_IM_END
        st = SlowArState.open(path, max_seq_len=96, device=rank, tp=(n, rank, nid))
        out = {}
        g = st.prefill(prompt.T.reshape(-1).astype(np.int32), logits="allowed", im_end_id=im_end)
        out["prefill"] = (g.hidden, g.logits)
        # teacher-forced steps on the engine's step program (exchange over NVLink)
        out["steps"] = [(r.hidden, r.logits) for r in
                        (st.step(s, logits="allowed", im_end_id=im_end) for s in steps)]
        res = generate_codes(st, im_end, st.graph_spec(), PromptTensor(prompt.shape[0], prompt.shape[1],
                                                                       prompt.reshape(-1)),
                             GenerateParams(frames, 0.0, 1.0, 0, 2 * frames + 2), FastArWeights.from_state(st),
                             SeededRng(0))
        out["codes"] = res.codes.reshape(-1, res.n_frames)
        st.close()
        q.put((rank, out, None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, repr(e)))


@pytest.mark.parametrize("n", [2, 4, 8])
@pytest.mark.parametrize("key", ["f16", "q4_k"])
def test_tp_engine_c2_shapes(n, key, model_dir):
    """n-way tensor parallelism on the persistent engine at C2's layer shapes:
    wo and w2 partial sums go straight into every rank's exchange buffer over
    NVLink and every rank sums them in rank order.  Ranks agree bit for bit;
    prefill, engine steps and greedy generation follow the oracle."""
    if n_gpus() < n:
        pytest.skip(f"needs {n} GPUs")
    import torch.multiprocessing as mp

    from fish_s2pro_b200 import nccl_unique_id, synth
    m = C2S_MODEL if key == "f16" else C5S_MODEL
    tol = 2e-2 if key == "f16" else 5e-2
    im_end = configs.S2PRO_IM_END
    path = synth.cached_gguf(m, model_dir)
    rng = np.random.default_rng(40 + n)
    prompt = np.zeros((m.num_codebooks + 1, 20), dtype=np.uint32)
    prompt[0] = rng.integers(0, m.sem_begin, size=20, dtype=np.uint32)
    cpu = o.OracleModel(str(path), max_seq_len=96, mode=0)
    try:
        h, lg = cpu.eval(prompt.T.reshape(-1).astype(np.int32), allowed_only=True, im_end_id=im_end)
        pre = (h, lg)
        steps, ref = [], []
        for i in range(2):
            main = m.sem_begin + int(np.argmax(lg[m.sem_begin:m.sem_end + 1]))
            steps.append([main, main - m.sem_begin] +
                         [int(c) for c in (np.arange(1, m.num_codebooks) * (41 + i)) % m.codebook_size])
            h, lg = cpu.eval(steps[-1], allowed_only=True, im_end_id=im_end)
            ref.append((h, lg))
        frames = 3
        nid = nccl_unique_id()
        ctx = mp.get_context("spawn")
        q = ctx.Queue()
        procs = [ctx.Process(target=_engine_rank, args=(r, n, nid, str(path), prompt, steps, frames, q))
                 for r in range(n)]
        for p in procs:
            p.start()
        res = {}
        try:
            for _ in procs:
                r, out, err = q.get(timeout=600)
                assert err is None, f"rank {r}: {err}"
                res[r] = out
        finally:
            for p in procs:
                p.join(timeout=60)
                if p.is_alive():
                    p.kill()
        for r in range(n):
            assert rel_err(res[r]["prefill"][1], pre[1]) < tol, r
            for i, (gh, gl) in enumerate(res[r]["steps"]):
                assert rel_err(gl, ref[i][1]) < tol, (r, i)
                assert rel_err(gh, ref[i][0]) < tol, (r, i)
            # the ranks sum the same partials in the same order
            for i in range(len(steps)):
                assert np.array_equal(res[r]["steps"][i][1], res[0]["steps"][i][1]), (r, i)
            assert np.array_equal(res[r]["codes"], res[0]["codes"]), r
        codes = res[0]["codes"]
        assert codes.shape == (m.num_codebooks, frames)
        cpu.reset()
        h, lg = cpu.eval(prompt.T.reshape(-1).astype(np.int32), allowed_only=True, im_end_id=im_end)
        for f in range(frames):
            assert greedy_consistent(int(codes[0, f]), lg[m.sem_begin:m.sem_end + 1], tol), f
            for k in range(1, m.num_codebooks):
                assert greedy_consistent(int(codes[k, f]), cpu.fast_prefix_logits(h, codes[:k, f].tolist()),
                                         tol), (f, k)
            h, lg = cpu.eval([m.sem_begin + int(codes[0, f])] + codes[:, f].tolist(), allowed_only=True,
                             im_end_id=im_end)
    finally:
        cpu.close()
