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
