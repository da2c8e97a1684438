"""Host side of Slow-AR tensor parallelism, on the CPU.

* s2d_tp_plan partitions the query heads, the KV heads and the FFN columns
  exactly (every head / column on one rank, whole weight blocks, GQA groups
  kept together) for the C1 and C2..C5 shapes and F16 / Q8_0 / Q4_K.
* Two gloo ranks run the sharded arithmetic of one Slow-AR layer the way the
  device path does (rank 0's wo / w2 outputs carry the residual, the others
  only their partial sums, then an allreduce) and match the unsharded layer.
"""
import os

import numpy as np
import pytest

from fish_s2pro_b200 import configs

UNIT = {configs.GGML_F16: 8, configs.GGML_Q8_0: 32, configs.GGML_Q4_K: 256}


def spec_of(m):
    from fish_s2pro_b200.s2d import GraphSpec
    return GraphSpec(slow_layers=m.slow_layers, hidden=m.d, ffn=m.ffn, heads=m.heads, kv_heads=m.kv_heads,
                     head_dim=m.head_dim, context_length=m.context_length, fast_layers=m.fast_layers,
                     fast_ffn=m.fast_ffn, fast_heads=m.fast_heads, fast_kv_heads=m.fast_kv_heads,
                     fast_head_dim=m.fast_head_dim, fast_context_length=m.num_codebooks + 1,
                     rope_base=1e6, rms_eps=1e-6, fast_rope_base=1e6, fast_rms_eps=1e-6,
                     codebook_size=m.codebook_size, num_codebooks=m.num_codebooks,
                     semantic_begin_id=m.sem_begin, semantic_end_id=m.sem_end, vocab_size=m.vocab,
                     codebook_rows=m.num_codebooks * m.codebook_size, linear_type=m.linear_type)


@pytest.mark.parametrize("lt", [configs.GGML_F16, configs.GGML_Q8_0, configs.GGML_Q4_K])
@pytest.mark.parametrize("model", ["tiny", "s2pro"])
def test_plan_partitions_heads_and_ffn(model, lt):
    from fish_s2pro_b200 import S2dError, tp_plan
    m = configs.tiny(linear_type=lt) if model == "tiny" else configs.s2pro(linear_type=lt)
    spec = spec_of(m)
    rep = m.heads // m.kv_heads
    for n in (1, 2, 4, 8):
        try:
            shards = [tp_plan(spec, n, r) for r in range(n)]
        except S2dError:
            # only when the heads or the FFN blocks cannot split n ways
            assert (m.kv_heads % n or (m.heads // n * m.head_dim) % UNIT[lt]
                    or m.ffn // UNIT[lt] < n), (model, lt, n)
            continue
        heads = [h for s in shards for h in range(s["head0"], s["head0"] + s["heads"])]
        kvh = [h for s in shards for h in range(s["kv_head0"], s["kv_head0"] + s["kv_heads"])]
        cols = [c for s in shards for c in range(s["ffn0"], s["ffn0"] + s["ffn"])]
        assert heads == list(range(m.heads)) and kvh == list(range(m.kv_heads))
        assert cols == list(range(m.ffn))
        for s in shards:
            assert s["ffn"] % UNIT[lt] == 0 and s["ffn0"] % UNIT[lt] == 0
            assert (s["head0"] * m.head_dim) % UNIT[lt] == 0
            # each query head's KV head (attention.rs:215-218) is on the same rank
            for h in range(s["head0"], s["head0"] + s["heads"]):
                assert s["kv_head0"] <= h // rep < s["kv_head0"] + s["kv_heads"]


def _layer_rank(rank, world, port, q):
    """One rank of the sharded FFN + attention-output arithmetic."""
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        from fish_s2pro_b200 import tp_plan
        m = configs.tiny()
        spec = spec_of(m)
        s = tp_plan(spec, world, rank)
        rng = np.random.default_rng(3)
        d, F, hd = m.d, m.ffn, m.head_dim
        x = rng.standard_normal(d).astype(np.float32)
        att = rng.standard_normal(m.heads * hd).astype(np.float32)
        wo = (rng.standard_normal((d, m.heads * hd)) * 0.02).astype(np.float32)
        w1 = (rng.standard_normal((F, d)) * 0.02).astype(np.float32)
        w3 = (rng.standard_normal((F, d)) * 0.02).astype(np.float32)
        w2 = (rng.standard_normal((d, F)) * 0.02).astype(np.float32)
        # the full layer (slow_ar.rs:659-710, 722-789): residual adds of wo and w2
        x1 = x + wo @ att
        g, u = w1 @ x1, w3 @ x1
        full = x1 + w2 @ ((g / (1 + np.exp(-g))) * u)
        # this rank's shard: its heads' attention columns, its FFN slice
        c0, c1 = s["head0"] * hd, (s["head0"] + s["heads"]) * hd
        part = wo[:, c0:c1] @ att[c0:c1] + (x if rank == 0 else 0)
        t = torch.from_numpy(part.astype(np.float32))
        dist.all_reduce(t)
        y1 = t.numpy()
        f0, f1 = s["ffn0"], s["ffn0"] + s["ffn"]
        g, u = w1[f0:f1] @ y1, w3[f0:f1] @ y1
        part = w2[:, f0:f1] @ ((g / (1 + np.exp(-g))) * u) + (y1 if rank == 0 else 0)
        t = torch.from_numpy(part.astype(np.float32))
        dist.all_reduce(t)
        q.put((rank, float(np.max(np.abs(t.numpy() - full)) / np.max(np.abs(full)))))
    finally:
        dist.destroy_process_group()


def test_sharded_layer_matches_unsharded_on_two_gloo_ranks():
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_layer_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0] < 1e-5 and res[1] < 1e-5, res
