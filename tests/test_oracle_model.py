"""Model-level oracle checks on the tiny C1 model (CPU only).

These pin the oracle's model code against the committed goldens and check the
equivalences the GPU path relies on: the Fast-AR with a KV cache equals the
reference's per-codebook prefix recomputation (fast_ar.rs:245-292, 360-437)
bit for bit, and computing only the unmasked LM-head rows leaves every sample
unchanged.
"""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from fish_s2pro_b200 import configs
from oracle import oracle as o

GOLDEN = json.loads((Path(__file__).parent / "golden" / "c1_oracle.json").read_text())


@pytest.fixture(scope="module")
def om(tiny_gguf):
    return o.OracleModel(tiny_gguf, max_seq_len=256, mode=0)


def test_synthetic_model_and_prompt_match_golden(tiny_gguf):
    assert hashlib.sha256(Path(tiny_gguf).read_bytes()).hexdigest() == GOLDEN["gguf_sha256"]
    p = configs.C1.prompt()
    assert hashlib.sha256(p.tobytes()).hexdigest() == GOLDEN["prompt_sha256"]


def test_graph_spec_reads_metadata(om):
    s = om.spec
    m = configs.C1.model
    assert (s.slow_block_count, s.slow_embedding_length, s.slow_head_count, s.slow_head_count_kv,
            s.slow_head_dim, s.slow_feed_forward_length) == (m.slow_layers, m.d, m.heads,
                                                               m.kv_heads, m.head_dim, m.ffn)
    assert s.fast_block_count == m.fast_layers and s.fast_head_dim == m.fast_head_dim
    assert s.vocab_size == m.vocab and s.num_codebooks == m.num_codebooks
    assert s.slow_attention_qk_norm == 1 and s.fast_attention_qk_norm == 0


def test_prefill_matches_golden(om):
    om.reset()
    flat = configs.C1.prompt().T.reshape(-1).astype(np.int32)
    hidden, logits = om.eval(flat)
    m = configs.C1.model
    assert hidden[:8].tolist() == pytest.approx(GOLDEN["prefill_hidden_first8"], abs=0)
    assert hashlib.sha256(logits.tobytes()).hexdigest() == GOLDEN["prefill_logits_sha256"]
    assert int(np.argmax(logits[m.sem_begin:m.sem_end + 1])) == GOLDEN["prefill_semantic_argmax"]


def test_decode_equals_prefill_at_model_level(om):
    """Prefilling n tokens at once equals prefilling n-1 then stepping one
    (slow_ar.rs:1454-1493 at layer level; here through all layers)."""
    m = configs.C1.model
    p = configs.C1.prompt()[:, :9].copy()
    p[0, 8] = m.sem_begin + 3
    p[1:, 8] = [1, 2, 3, 4]
    flat = p.T.reshape(-1).astype(np.int32)
    om.reset()
    h_all, l_all = om.eval(flat)
    om.reset()
    om.eval(flat[:-5])
    h_step, l_step = om.eval(flat[-5:])
    assert np.array_equal(h_all, h_step) and np.array_equal(l_all, l_step)
    assert om.n_past() == 9


def test_eval_rejects_bad_width_and_overflow(tiny_gguf):
    small = o.OracleModel(tiny_gguf, max_seq_len=4, mode=0)
    with pytest.raises(o.OracleError, match="not a multiple of codebook_dim"):
        small.eval(np.zeros(7, np.int32))
    with pytest.raises(o.OracleError, match="KV cache overflow"):
        small.eval(np.zeros(5 * 5, np.int32))


def test_fast_prefix_matches_golden(om):
    om.reset()
    flat = configs.C1.prompt().T.reshape(-1).astype(np.int32)
    hidden, _ = om.eval(flat, logits=False)
    lg = om.fast_prefix_logits(hidden, [5, 17])
    assert lg[:8].tolist() == pytest.approx(GOLDEN["fast_prefix_5_17_first8"], abs=0)
    with pytest.raises(o.OracleError, match="fast prefix too long"):
        om.fast_prefix_logits(hidden, [1, 2, 3, 4])


def test_generate_codes_matches_golden(om):
    codes, mains = om.generate_codes(configs.C1.prompt(), GOLDEN["greedy_params"], o.SeededRng(0))
    assert codes.tolist() == GOLDEN["greedy_codes"]
    assert mains.tolist() == GOLDEN["greedy_main_tokens"]
    codes, mains = om.generate_codes(configs.C1.prompt(), GOLDEN["sampled_params"],
                                     o.SeededRng(GOLDEN["sampled_seed"]))
    assert codes.tolist() == GOLDEN["sampled_codes"]
    assert mains.tolist() == GOLDEN["sampled_main_tokens"]


def test_faithful_mode_is_bit_identical(tiny_gguf, om):
    """Reference-faithful mode (full-vocab LM head, per-step f32 re-expansion,
    Fast-AR prefix recomputation) gives the same codes and RNG stream."""
    faithful = o.OracleModel(tiny_gguf, max_seq_len=256, mode=1)
    params = dict(GOLDEN["sampled_params"])
    a = om.generate_codes(configs.C1.prompt(), params, o.SeededRng(77))
    b = faithful.generate_codes(configs.C1.prompt(), params, o.SeededRng(77))
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    om.reset()
    faithful.reset()
    flat = configs.C1.prompt().T.reshape(-1).astype(np.int32)
    ha, _ = om.eval(flat, logits=False)
    hb, _ = faithful.eval(flat, logits=False)
    assert np.array_equal(ha, hb)
    for prefix in ([3], [3, 9], [3, 9, 1000]):
        assert np.array_equal(om.fast_prefix_logits(ha, prefix),
                              faithful.fast_prefix_logits(hb, prefix))


def test_allowed_rows_equal_full_rows(om):
    m = configs.C1.model
    flat = configs.C1.prompt().T.reshape(-1).astype(np.int32)
    om.reset()
    _, full = om.eval(flat)
    om.reset()
    _, allowed = om.eval(flat, allowed_only=True, im_end_id=configs.C1.im_end_id)
    sl = slice(m.sem_begin, m.sem_end + 1)
    assert np.array_equal(full[sl], allowed[sl])
    assert full[configs.C1.im_end_id] == allowed[configs.C1.im_end_id]
    mask = np.ones(m.vocab, bool)
    mask[sl] = False
    mask[configs.C1.im_end_id] = False
    assert np.all(np.isneginf(allowed[mask]))


def test_thread_count_does_not_change_results(om):
    flat = configs.C1.prompt().T.reshape(-1).astype(np.int32)
    n0 = o.get_threads()
    try:
        o.set_threads(1)
        om.reset()
        h1, l1 = om.eval(flat)
        o.set_threads(max(n0, 3))
        om.reset()
        h3, l3 = om.eval(flat)
    finally:
        o.set_threads(n0)
    assert np.array_equal(h1, h3) and np.array_equal(l1, l3)
