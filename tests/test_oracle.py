"""The CPU oracle against the reference's golden fixture and unit-test known answers.

These tests pin the oracle before any CUDA result is compared with it.
"""
import json
import math
import os

import numpy as np
import pytest

from oracle.model import (OracleModel, WeDLMConfig, apply_rope, bf16_round, random_weights,
                          rms_norm, rope_tables)
from oracle.sampler import (SamplingParams, compute_entropies_with_probs, effective_cap,
                            greedy_argmax_last, row_stats, select_by_entropy_with_distance,
                            update_running_entropy)
from oracle.decoder import (OracleDecoder, compute_block_reorder, topological_reorder_cpu)

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def load_ref_fixture():
    with open(os.path.join(GOLDEN, "ref_parity_small.json")) as f:
        fx = json.load(f)
    cfg = WeDLMConfig.from_dict(fx["config"])
    w = {k: np.asarray(v["data"], np.float32).reshape(v["shape"]) for k, v in fx["weights"].items()}
    exp = np.asarray(fx["expected_logits"]["data"], np.float32).reshape(fx["expected_logits"]["shape"])
    return fx, cfg, w, exp


def test_ref_fixture_explicit_positions():
    """tests/parity_explicit_positions.rs:73-128 (tolerance there: 1e-3)."""
    fx, cfg, w, exp = load_ref_fixture()
    m = OracleModel(cfg, w, "f32")
    logits, _ = m.forward_with_positions(fx["input_ids"][0], fx["positions"][0])
    err = np.abs(logits - exp[0]).max()
    assert err < 1e-5, err


def test_ref_fixture_cache_consistency():
    """Prefix-cache consistency (the idea of tests/invariant_tests.rs:649-712): running
    the same tokens as prefix-cache + block gives the same logits as one forward."""
    fx, cfg, w, _ = load_ref_fixture()
    m = OracleModel(cfg, w, "f32")
    ids, pos = fx["input_ids"][0], fx["positions"][0]
    full, _ = m.forward_with_positions(ids, pos)
    _, cache = m.forward_with_positions(ids[:2], pos[:2])
    tail, _ = m.forward_with_positions(ids[2:], pos[2:], cache)
    assert np.abs(full[2:] - tail).max() < 1e-6


# --- sampler.rs:547-610 known answers ------------------------------------------------
def test_select_by_entropy_with_distance_known_answer():
    sel = select_by_entropy_with_distance([0.3, 0.1, 0.5, 0.2], [10, 11, 12, 13], 0.4, 0.1, 10)
    assert sorted(sel) == [0, 1]


def test_distance_penalty_biases_left():
    sel = select_by_entropy_with_distance([0.3] * 4, [5, 6, 7, 8], 0.5, 0.1, 2)
    assert sorted(sel) == [0, 1]


def test_fallback_to_min_entropy():
    assert select_by_entropy_with_distance([0.8, 0.9, 0.7], [0, 1, 2], 0.3, 0.0, 10) == [2]


def test_fallback_first_minimum_and_cap_order():
    # ties in adjusted entropy: the FIRST in logical order wins (Iterator::min_by)
    assert select_by_entropy_with_distance([0.9, 0.9, 0.9], [7, 3, 5], 0.1, 0.0, 4) == [1]
    # selection is in ascending logical order, truncated to the cap (not lowest entropy)
    sel = select_by_entropy_with_distance([0.1, 0.0, 0.2, 0.05], [3, 1, 2, 0], 1.0, 0.0, 2)
    assert sel == [3, 1]
    assert select_by_entropy_with_distance([], [], 1.0, 0.0, 2) == []


# --- reorder.rs:194-253 known answers ------------------------------------------------
def test_topological_reorder_cpu():
    ids, perm, inv, nk = topological_reorder_cpu([1, 151666, 2, 151666], [1, 3])
    assert nk == 2 and perm == [0, 2, 1, 3] and ids == [1, 2, 151666, 151666]


def test_reorder_ignores_token_value():
    _, perm, _, nk = topological_reorder_cpu([1, 151666, 2, 151666], [3])
    assert nk == 3 and perm == [0, 1, 2, 3]


def test_compute_block_reorder():
    r = compute_block_reorder([100, 200, 151666, 151666], [2, 3], 10)
    assert r.num_filled == 2 and r.reordered_block == [100, 200, 151666, 151666]
    assert r.positions == [10, 11, 12, 13] and r.block_permutation == [0, 1, 2, 3]


def test_compute_block_reorder_mixed():
    r = compute_block_reorder([151666, 100, 151666, 200], [0, 2], 5)
    assert r.num_filled == 2 and r.reordered_block == [100, 200, 151666, 151666]
    assert r.positions == [6, 8, 5, 7] and r.block_permutation == [1, 3, 0, 2]


# --- rope.rs:204-246, attention.rs:336-368, mlp.rs:52-69, config.rs:157-165 --------
def test_rope_inv_freq_and_shape():
    cos, sin = rope_tables(128, 16, 1_000_000.0, False)
    assert cos.shape == (16, 64) and sin.shape == (16, 64)
    # position 1 row = inv_freq
    assert abs(cos[1, 0] - math.cos(1.0)) < 1e-6
    assert math.acos(cos[1, 63]) < 0.01


def test_rms_norm_sanity():
    y = rms_norm(np.array([[1, 2, 3, 4]], np.float32), np.ones(4, np.float32), 1e-6)
    assert 0 < y[0, 0] < 1
    assert abs(y[0, 3] - 4 / math.sqrt(7.5)) < 1e-5


def test_causal_mask_upper_triangle():
    cfg = WeDLMConfig(vocab_size=8, hidden_size=8, num_hidden_layers=1, num_attention_heads=2,
                      num_key_value_heads=1, head_dim=4, intermediate_size=8,
                      max_position_embeddings=16, dtype="float32")
    w = random_weights(cfg, 1, 0.5)
    m = OracleModel(cfg, w, "f32")
    # query 0 must not see keys 1, 2: changing tokens 1..2 leaves row 0 unchanged
    a, _ = m.forward_with_positions([1, 2, 3], [0, 1, 2])
    b, _ = m.forward_with_positions([1, 5, 6], [0, 1, 2])
    assert np.abs(a[0] - b[0]).max() == 0
    assert np.abs(a[2] - b[2]).max() > 0


def test_silu_values():
    x = np.array([0.0, 1.0, -1.0], np.float32)
    s = x / (1 + np.exp(-x))
    assert abs(s[0]) < 1e-6 and abs(s[1] - 0.731) < 0.01 and abs(s[2] + 0.269) < 0.01


def test_wedlm_8b_config():
    c = WeDLMConfig.wedlm_8b()
    assert c.num_kv_groups == 4 and c.head_dim == 128 and c.qk_norm and c.rope_theta == 1e6


# --- entropy / argmax restatement -----------------------------------------------------
def test_entropy_and_argmax_last_max():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((5, 1000)).astype(np.float32) * 2.5
    x[1, 10] = x[1, 900] = x[1].max() + 1.0  # tie: last index wins
    H, p = compute_entropies_with_probs(x, 0.0)
    H2, am, mp = row_stats(x, 0.0)
    assert np.allclose(H, H2, atol=1e-5)
    assert am[1] == 900 and greedy_argmax_last(p[1]) == 900
    assert np.allclose(mp, p.max(axis=1), rtol=1e-6)
    # temperature scaling only when T not in {0, 1}
    Ht, _ = compute_entropies_with_probs(x, 0.5)
    assert np.allclose(Ht, compute_entropies_with_probs(x * 2, 1.0)[0], atol=1e-5)


def test_entropy_ema_cap():
    r = update_running_entropy(0.8, [0.0, 0.0])
    assert abs(r - 0.56) < 1e-6
    assert effective_cap(0.2, 0.8, 8) == 16
    assert effective_cap(0.5, 0.8, 8) == 12
    assert effective_cap(0.7, 0.8, 6) == 6
    assert effective_cap(0.5, 0.8, 7) == 11


def test_bf16_round():
    x = np.array([1.0, 1.00390625, 1.005859375, -3.14159, 0.0], np.float32)
    r = bf16_round(x)
    assert r[0] == 1.0 and r[1] == 1.0  # tie to even
    assert r[2] == 1.0078125
    assert abs(r[3] + 3.140625) < 1e-7


# --- streaming loop semantics ----------------------------------------------------------
class _ScriptedModel:
    """A fake model whose logits make chosen rows confident (for branch coverage)."""

    def __init__(self, V, confident):
        self.V, self.confident = V, confident
        self.calls = []

    def prefill_cache(self, ids):
        z = np.zeros((1, len(ids), 1), np.float32)
        return [(z, z)]

    def forward_with_positions(self, ids, pos, cache):
        self.calls.append((list(ids), list(pos)))
        blk = np.zeros((1, len(ids), 1), np.float32)
        cache = [(np.concatenate([k, blk], 1), np.concatenate([v, blk], 1)) for k, v in cache]
        S = len(ids)
        lg = np.zeros((S, self.V), np.float32)
        for i, p in enumerate(pos):
            tok = (p * 7) % (self.V - 2) + 1
            lg[i, tok] = 30.0 if p in self.confident else 0.5
        return lg, cache


def test_streaming_commit_before_predict_and_refill():
    V = 64
    model = _ScriptedModel(V, confident={10, 11, 12})
    dec = OracleDecoder(model, mask_token_id=V - 1, eos_token_id=10_000)
    params = SamplingParams(temperature=0.0, entropy_threshold=0.8, distance_penalty=0.05,
                            max_tokens_per_step=8)
    ids, st = dec.generate_streaming(list(range(10)), 6, 4, params)
    out = ids[10:]
    assert len(out) == 6
    assert out == [(p * 7) % (V - 2) + 1 for p in range(10, 16)]
    # step 1: whole window masked, confident slots 10, 11, 12 selected together
    assert dec.trace[0].selected == [0, 1, 2] and dec.trace[0].n_commit == 0
    # step 2: the three filled tokens are committed (commit-before-predict)
    assert dec.trace[1].n_commit == 3
    # reordered: filled first, masks last, with true positions
    assert dec.trace[1].reordered_positions[:3] == [10, 11, 12]


# --- the C restatement (CPU baseline / checker) against the numpy restatement ------
def test_c_restatement_matches_numpy():
    from oracle import cbind
    from oracle.model import f32_to_bf16_bits, bf16_bits_to_f32
    rng = np.random.default_rng(0)
    x = rng.standard_normal((24, 20000), dtype=np.float32) * 2.5
    x[3, 7] = 40.0
    b = f32_to_bf16_bits(x)
    mask_pos = rng.permutation(30)[:24].tolist()
    r = cbind.entropy_select(b, "bf16", 0.0, 0.8, 0.05, [0, 10, 24], mask_pos, [8, 2])
    H, am, _ = row_stats(bf16_bits_to_f32(b), 0.0)
    # the reference sums p ln p sequentially in f32: ~1e-4 from the exact value here
    assert np.abs(r["H"] - H).max() < 2e-3
    assert (r["tokens"] == am).all()
    for s, (r0, r1, cap) in enumerate([(0, 10, 8), (10, 24, 2)]):
        want = select_by_entropy_with_distance(r["H"][r0:r1].tolist(), mask_pos[r0:r1], 0.8, 0.05, cap)
        assert r["selected"][r0:r0 + r["n_selected"][s]].tolist() == want
    # f32 input and temperature scaling
    rf = cbind.entropy_select(x, "f32", 0.5, 0.8, 0.05, [0, 24], mask_pos, [8])
    Hf, amf, _ = row_stats(x, 0.5)
    assert np.abs(rf["H"] - Hf).max() < 2e-3 and (rf["tokens"] == amf).all()


def test_seeded_sampling_restatement():
    """sample_from_probs / sample_nucleus (sampler.rs:306-351) with the draw given, and
    the SplitMix64 draws: known answers, the nucleus bound, and frequencies that follow
    the probabilities."""
    from oracle.sampler import sample_from_probs, sample_nucleus, sampling_uniform, splitmix64
    # SplitMix64 reference outputs for state 0 (the generator's first three outputs)
    assert splitmix64(0) == 0xE220A8397B1DCDAF
    p = np.array([0.1, 0.4, 0.2, 0.3], np.float32)
    assert [sample_from_probs(p, r) for r in (0.05, 0.12, 0.49, 0.51, 0.71, 0.99)] == [0, 1, 1, 2, 3, 3]
    # nucleus at 0.6: tokens 1 (0.4) and 3 (0.3), renormalised over 0.7
    assert [sample_nucleus(p, 0.6, r) for r in (0.0, 0.5, 0.57, 0.58, 0.99)] == [1, 1, 1, 3, 3]
    # ties keep index order: 2 and 3 tie, 2 comes first
    q = np.array([0.1, 0.3, 0.3, 0.3], np.float32)
    assert sample_nucleus(q, 0.5, 0.2) == 1 and sample_nucleus(q, 0.5, 0.8) == 2
    u = np.array([sampling_uniform(7, 0, s, i) for s in range(1, 41) for i in range(50)])
    assert u.min() >= 0.0 and u.max() < 1.0 and abs(u.mean() - 0.5) < 0.02
    assert len(set(u.tolist())) > 1990
    probs = np.array([0.05, 0.5, 0.15, 0.3])
    counts = np.bincount([sample_from_probs(probs, x) for x in u], minlength=4) / len(u)
    assert np.abs(counts - probs).max() < 0.02
    nuc = [sample_nucleus(probs, 0.7, x) for x in u]
    assert set(nuc) == {1, 3}
    assert abs(np.mean(np.array(nuc) == 1) - 0.5 / 0.8) < 0.03
