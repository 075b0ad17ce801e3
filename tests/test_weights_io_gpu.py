"""wedlm_load_weights: safetensors checkpoints (single file, or shards with
model.safetensors.index.json) as src/weights.rs:27-210 reads them.

The oracle's weights are written to disk with the test writer (tests/safetensors_io.py)
and loaded through the C ABI; every stored tensor must equal the one uploaded through
wedlm_set_weight (bit-exact: both paths convert on the host the same way), the logits of
a forward must be identical, and missing files / tensors and malformed headers must
fail with NOT_FOUND / IO.
"""
import json
import os
import struct

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle.model import random_weights
from model_configs import c1_config, long_ctx_bf16_config, to_model_config
from safetensors_io import write_safetensors, write_sharded

ERR_NOT_FOUND, ERR_IO = -5, -6


def make_ctx(cfg):
    from wedlm_b200 import Context
    return Context(to_model_config(cfg, max_block_tokens=32), max_seqs=1, max_ctx=128)


def forward_logits(ctx, cfg):
    rng = np.random.default_rng(4)
    ctx.reset_sequence(0)
    ctx.prefill(0, rng.integers(0, cfg.vocab_size - 2, size=20))
    win = rng.integers(0, cfg.vocab_size - 2, size=16)
    return ctx.forward_with_positions([0], win[None], np.arange(20, 36)[None],
                                      logits_dtype=torch.float32).cpu().numpy()


def shapes(w):
    return {k: v.shape for k, v in w.items()}


def test_single_file_f32_matches_set_weight(tmp_path):
    cfg = c1_config()
    w = random_weights(cfg, seed=0, std=0.02)
    write_safetensors(tmp_path / "model.safetensors", w)
    a, b = make_ctx(cfg), make_ctx(cfg)
    try:
        a.load_safetensors(tmp_path)
        b.load_weights(w)
        for k, s in shapes(w).items():
            assert np.array_equal(a.get_weight(k, s), b.get_weight(k, s)), k
        assert np.array_equal(forward_logits(a, cfg), forward_logits(b, cfg))
    finally:
        a.close()
        b.close()


def test_sharded_bf16_with_extra_tensor(tmp_path):
    cfg = long_ctx_bf16_config()
    w = random_weights(cfg, seed=1, std=0.02)
    extra = dict(w)
    extra["model.rotary_emb.inv_freq"] = np.ones(64, np.float32)  # not a model tensor
    write_sharded(str(tmp_path), extra, nshards=3, bf16=True)
    a, b = make_ctx(cfg), make_ctx(cfg)
    try:
        a.load_safetensors(tmp_path)
        b.load_weights(w)
        for k, s in shapes(w).items():
            assert np.array_equal(a.get_weight(k, s), b.get_weight(k, s)), k
        assert np.array_equal(forward_logits(a, cfg), forward_logits(b, cfg))
    finally:
        a.close()
        b.close()


def test_f16_and_f64_tensors(tmp_path):
    cfg = c1_config()
    w = random_weights(cfg, seed=2, std=0.02)
    mixed = dict(w)
    mixed["model.norm.weight"] = w["model.norm.weight"].astype(np.float64) * 1.5
    q = "model.layers.0.self_attn.q_proj.weight"
    mixed[q] = w[q].astype(np.float16)
    write_safetensors(tmp_path / "model.safetensors", mixed)
    ctx = make_ctx(cfg)
    try:
        ctx.load_safetensors(tmp_path)
        assert np.array_equal(ctx.get_weight("model.norm.weight", (cfg.hidden_size,)),
                              (w["model.norm.weight"].astype(np.float64) * 1.5).astype(np.float32))
        assert np.array_equal(ctx.get_weight(q, w[q].shape),
                              w[q].astype(np.float16).astype(np.float32))
    finally:
        ctx.close()


def test_missing_and_malformed(tmp_path):
    from wedlm_b200 import WedlmError
    cfg = c1_config()
    w = random_weights(cfg, seed=3, std=0.02)
    ctx = make_ctx(cfg)
    try:
        with pytest.raises(WedlmError) as e:
            ctx.load_safetensors(tmp_path)  # empty directory
        assert e.value.code == ERR_NOT_FOUND
        partial = {k: v for k, v in w.items() if k != "model.norm.weight"}
        write_safetensors(tmp_path / "model.safetensors", partial)
        with pytest.raises(WedlmError) as e:
            ctx.load_safetensors(tmp_path)
        assert e.value.code == ERR_NOT_FOUND and "model.norm.weight" in str(e.value)
        # header length past the end of the file
        with open(tmp_path / "model.safetensors", "wb") as f:
            f.write(struct.pack("<Q", 1 << 40) + b"{}")
        with pytest.raises(WedlmError) as e:
            ctx.load_safetensors(tmp_path)
        assert e.value.code == ERR_IO
        # data_offsets that do not match the shape
        hdr = json.dumps({"model.norm.weight": {"dtype": "F32", "shape": [cfg.hidden_size],
                                                "data_offsets": [0, 8]}}).encode()
        with open(tmp_path / "model.safetensors", "wb") as f:
            f.write(struct.pack("<Q", len(hdr)) + hdr + b"\0" * 8)
        with pytest.raises(WedlmError) as e:
            ctx.load_safetensors(tmp_path)
        assert e.value.code == ERR_IO
    finally:
        ctx.close()
