"""Numpy restatement of ``WeDLMForCausalLM`` (test infrastructure only).

Follows the reference forward path:

* embedding gather            ``src/model/backbone.rs:37-58``
* RMSNorm (f32 math, x/sqrt)  ``src/model/attention.rs:35-50``
* q/k/v/o projections         ``src/model/attention.rs:90-93,145-147,229``
* QK-norm before transpose    ``src/model/attention.rs:154-163``
* RoPE, rotate-half, explicit positions
                              ``src/model/rope.rs:37-97,132-146,158-197``
* KV concat (cache ++ block)  ``src/model/attention.rs:173-184``
* causal mask over the reordered index (query i sees every cached key and the block
  keys with index <= i)       ``src/model/attention.rs:255-279`` via
                              ``src/model/backbone.rs:158-178``
* attention (GQA repeat_kv)   ``src/model/attention.rs:188-199,238-249``
* SwiGLU MLP                  ``src/model/mlp.rs:38-45``
* pre-norm residual layer     ``src/model/layer.rs:58-81``
* final norm + LM head on all rows
                              ``src/model/backbone.rs:196``, ``src/model/causal_lm.rs:68-79``

``dtype='f32'`` is the exact fp32 computation of the reference with an f32 model.
``dtype='bf16'`` keeps f32 arithmetic but rounds to bf16 at the points where a bf16
B200 build stores tensors (weights, activations between kernels, the K/V cache, the
cos/sin table as in ``rope.rs:94-95``, logits).  It is the comparison point for the
bf16 kernels under the tolerances stated in the tests.

The ``rank`` argument generalises the mask: block key j is visible to block query i
iff ``rank[j] <= rank[i]``.  ``rank = arange(S)`` (the default) is the reference's
reordered-index causal mask; ``rank = positions`` is "causal over explicit
positions".
"""
from __future__ import annotations

import json
import math
from dataclasses import dataclass, field, asdict
from typing import Dict, List, Optional, Tuple

import numpy as np


def bf16_round(x) -> np.ndarray:
    """Round f32 values to the nearest bf16 (ties to even) and return them as f32."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    nan = np.isnan(x)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def f32_to_bf16_bits(x) -> np.ndarray:
    """f32 -> raw bf16 bit patterns (uint16), round to nearest even."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


@dataclass
class WeDLMConfig:
    """Shape/eps fields of ``WeDLMConfig`` (``src/config.rs:9-78``)."""

    vocab_size: int
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    intermediate_size: int
    max_position_embeddings: int = 16384
    rope_theta: float = 1_000_000.0
    rms_norm_eps: float = 1e-6
    qk_norm: bool = True
    eos_token_id: int = 0
    mask_token_id: Optional[int] = None
    dtype: str = "bfloat16"

    @staticmethod
    def wedlm_8b() -> "WeDLMConfig":
        """``WeDLMConfig::wedlm_8b`` (``src/config.rs:127-150``)."""
        return WeDLMConfig(vocab_size=151936, hidden_size=4096, num_hidden_layers=36,
                           num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                           intermediate_size=12288, max_position_embeddings=16384,
                           rope_theta=1_000_000.0, rms_norm_eps=1e-6, qk_norm=True,
                           eos_token_id=151643, mask_token_id=151666, dtype="bfloat16")

    @staticmethod
    def from_dict(d: dict) -> "WeDLMConfig":
        keys = WeDLMConfig.__dataclass_fields__.keys()
        return WeDLMConfig(**{k: d[k] for k in keys if k in d})

    def to_dict(self) -> dict:
        return asdict(self)

    @property
    def num_kv_groups(self) -> int:
        return self.num_attention_heads // self.num_key_value_heads


def weight_names(cfg: WeDLMConfig) -> List[Tuple[str, Tuple[int, ...]]]:
    """Tensor names and shapes in the reference's safetensors layout
    (``src/model/causal_lm.rs:23-31``, ``backbone.rs:76-100``, ``layer.rs:29-43``,
    ``attention.rs:83-103``, ``mlp.rs:20-31``)."""
    H, I, V = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size
    qd = cfg.num_attention_heads * cfg.head_dim
    kd = cfg.num_key_value_heads * cfg.head_dim
    out = [("model.embed_tokens.weight", (V, H))]
    for l in range(cfg.num_hidden_layers):
        p = f"model.layers.{l}."
        out += [
            (p + "input_layernorm.weight", (H,)),
            (p + "self_attn.q_proj.weight", (qd, H)),
            (p + "self_attn.k_proj.weight", (kd, H)),
            (p + "self_attn.v_proj.weight", (kd, H)),
            (p + "self_attn.o_proj.weight", (H, qd)),
        ]
        if cfg.qk_norm:
            out += [(p + "self_attn.q_norm.weight", (cfg.head_dim,)),
                    (p + "self_attn.k_norm.weight", (cfg.head_dim,))]
        out += [
            (p + "post_attention_layernorm.weight", (H,)),
            (p + "mlp.gate_proj.weight", (I, H)),
            (p + "mlp.up_proj.weight", (I, H)),
            (p + "mlp.down_proj.weight", (H, I)),
        ]
    out += [("model.norm.weight", (H,)), ("lm_head.weight", (V, H))]
    return out


def random_weights(cfg: WeDLMConfig, seed: int = 0, std: float = 0.02) -> Dict[str, np.ndarray]:
    """Seeded random init: linear/embedding weights N(0, std^2), norm weights ones.

    Drawn in ``weight_names`` order from ``numpy.random.default_rng(seed)``.
    """
    rng = np.random.default_rng(seed)
    w = {}
    for name, shape in weight_names(cfg):
        if name.endswith("norm.weight"):
            w[name] = np.ones(shape, np.float32)
        else:
            w[name] = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)
    return w


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """``RMSNorm::forward`` (``src/model/attention.rs:35-50``): f32 math,
    ``x / sqrt(mean(x^2) + eps) * w``."""
    x = x.astype(np.float32)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    y = x / np.sqrt(var + np.float32(eps))
    return (y * w.astype(np.float32)).astype(np.float32)


def rope_tables(head_dim: int, max_pos: int, theta: float, bf16: bool) -> Tuple[np.ndarray, np.ndarray]:
    """``RotaryEmbedding::new`` (``src/model/rope.rs:37-97``): inverse frequencies in
    f64 cast to f32, ``freqs = positions x inv_freq`` in f32, cos/sin cast to the
    model dtype.  Returns ``[max_pos, head_dim/2]`` tables."""
    half = head_dim // 2
    inv = np.array([np.float32(1.0 / math.pow(theta, (2 * i) / head_dim)) for i in range(half)],
                   dtype=np.float32)
    pos = np.arange(max_pos, dtype=np.float32)[:, None]
    freqs = (pos * inv[None, :]).astype(np.float32)
    cos = np.cos(freqs).astype(np.float32)
    sin = np.sin(freqs).astype(np.float32)
    if bf16:
        cos, sin = bf16_round(cos), bf16_round(sin)
    return cos, sin


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Rotate-half RoPE (``candle_nn::rotary_emb::rope`` as called from
    ``src/model/rope.rs:185-194``; same formula as
    ``scripts/generate_parity_fixture.py:42-59``).  ``x``: ``[heads, S, d]``,
    ``cos``/``sin``: ``[S, d/2]``."""
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    c, s = cos[None], sin[None]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1).astype(np.float32)


def softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
    m = np.max(x, axis=axis, keepdims=True)
    e = np.exp((x - m).astype(np.float32))
    return (e / np.sum(e, axis=axis, keepdims=True, dtype=np.float32)).astype(np.float32)


class _WeightStore:
    """Weights by name.  f32 arrays are rounded once at construction (bf16 mode);
    uint16 arrays are bf16 bit patterns kept as they are and widened to f32 on each
    access (exact: every bf16 value is an f32 value), so that a model with billions of
    parameters is held at two bytes per weight."""

    def __init__(self, weights: Dict[str, np.ndarray], rnd):
        self._a = {}
        for k, v in weights.items():
            v = np.asarray(v)
            self._a[k] = v if v.dtype == np.uint16 else rnd(v)

    def __getitem__(self, name: str) -> np.ndarray:
        v = self._a[name]
        return bf16_bits_to_f32(v) if v.dtype == np.uint16 else v

    def rows(self, name: str, idx) -> np.ndarray:
        """Rows ``idx`` of a matrix, widened after the gather."""
        v = self._a[name][np.asarray(idx)]
        return bf16_bits_to_f32(v) if v.dtype == np.uint16 else v

    def row_block(self, name: str, r0: int, r1: int) -> np.ndarray:
        v = self._a[name][r0:r1]
        return bf16_bits_to_f32(v) if v.dtype == np.uint16 else v

    def shape(self, name: str):
        return self._a[name].shape

    def keys(self):
        return self._a.keys()


class OracleModel:
    """``WeDLMForCausalLM`` restated in numpy.

    ``cache`` is a list (one per layer) of ``(K, V)`` with shape ``[n_kv, L, d]``;
    K is stored post-QK-norm, post-RoPE, V raw (``attention.rs:154-184``).
    ``weights`` values are f32 arrays, or uint16 arrays of bf16 bit patterns (held as
    such; see ``_WeightStore``).
    """

    LM_HEAD_CHUNK = 16384  # vocabulary rows per LM-head product (bounds the f32 copy)

    def __init__(self, cfg: WeDLMConfig, weights: Dict[str, np.ndarray], dtype: str = "f32"):
        assert dtype in ("f32", "bf16")
        self.cfg = cfg
        self.dtype = dtype
        rnd = bf16_round if dtype == "bf16" else (lambda a: np.asarray(a, np.float32))
        self._r = rnd
        self.w = _WeightStore(weights, rnd)
        self.cos, self.sin = rope_tables(cfg.head_dim, cfg.max_position_embeddings,
                                         cfg.rope_theta, dtype == "bf16")

    def _lm_head(self, h: np.ndarray) -> np.ndarray:
        """``h @ lm_head.T`` (``causal_lm.rs:77``) in vocabulary chunks, f32 accumulate."""
        V = self.w.shape("lm_head.weight")[0]
        out = np.empty((h.shape[0], V), np.float32)
        for v0 in range(0, V, self.LM_HEAD_CHUNK):
            v1 = min(V, v0 + self.LM_HEAD_CHUNK)
            out[:, v0:v1] = np.matmul(h, self.w.row_block("lm_head.weight", v0, v1).T,
                                      dtype=np.float32)
        return out

    # -- helpers ---------------------------------------------------------------
    def _lin(self, x, name):
        return self._r(np.matmul(x, self.w[name].T, dtype=np.float32))

    def _layer(self, l, h, positions, cache_kv, rank, want_logits_rows=None):
        cfg, r = self.cfg, self._r
        p = f"model.layers.{l}."
        S = h.shape[0]
        nh, nkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        x = r(rms_norm(h, self.w[p + "input_layernorm.weight"], cfg.rms_norm_eps))
        q = self._lin(x, p + "self_attn.q_proj.weight").reshape(S, nh, d)
        k = self._lin(x, p + "self_attn.k_proj.weight").reshape(S, nkv, d)
        v = self._lin(x, p + "self_attn.v_proj.weight").reshape(S, nkv, d)
        if cfg.qk_norm:
            q = r(rms_norm(q, self.w[p + "self_attn.q_norm.weight"], cfg.rms_norm_eps))
            k = r(rms_norm(k, self.w[p + "self_attn.k_norm.weight"], cfg.rms_norm_eps))
        q, k, v = q.transpose(1, 0, 2), k.transpose(1, 0, 2), v.transpose(1, 0, 2)
        cos, sin = self.cos[positions], self.sin[positions]
        q, k = r(apply_rope(q, cos, sin)), r(apply_rope(k, cos, sin))
        if cache_kv is not None:
            K = np.concatenate([cache_kv[0], k], axis=1)
            V = np.concatenate([cache_kv[1], v], axis=1)
        else:
            K, V = k, v
        L = K.shape[1] - S
        # mask: prefix always visible; block key j visible iff rank[j] <= rank[i]
        vis = np.ones((S, L + S), dtype=bool)
        vis[:, L:] = rank[None, :] <= rank[:, None]
        g = cfg.num_kv_groups
        Ke = np.repeat(K, g, axis=0)
        Ve = np.repeat(V, g, axis=0)
        scale = np.float32(1.0 / math.sqrt(d))
        sc = np.matmul(q, Ke.transpose(0, 2, 1), dtype=np.float32) * scale
        sc = np.where(vis[None], sc, np.float32(-np.inf))
        pr = softmax(sc, axis=-1)
        o = np.matmul(pr, Ve, dtype=np.float32)
        o = r(o).transpose(1, 0, 2).reshape(S, nh * d)
        h = r(h + self._lin(o, p + "self_attn.o_proj.weight"))
        x = r(rms_norm(h, self.w[p + "post_attention_layernorm.weight"], cfg.rms_norm_eps))
        gte = self._lin(x, p + "mlp.gate_proj.weight")
        up = self._lin(x, p + "mlp.up_proj.weight")
        act = r(gte / (np.float32(1.0) + np.exp(-gte)) * up)
        h = r(h + self._lin(act, p + "mlp.down_proj.weight"))
        return h, (K, V)

    # -- public API mirroring causal_lm.rs --------------------------------------
    def forward_with_positions(self, input_ids, positions, kv_caches=None, rank=None,
                               logits_rows: Optional[slice] = None, round_logits: bool = True,
                               return_hidden: bool = False):
        """``WeDLMForCausalLM::forward_with_positions`` (``causal_lm.rs:68-79``).

        Returns ``(logits [S or rows, V], new_caches)``.  ``new_caches`` holds the
        concatenated ``cache ++ block`` K/V per layer, as the reference returns.
        ``return_hidden`` returns the final-normed hidden rows (the LM head's input,
        ``causal_lm.rs:77``) in place of the logits.
        """
        ids = np.asarray(input_ids, dtype=np.int64).reshape(-1)
        pos = np.asarray(positions, dtype=np.int64).reshape(-1)
        if pos.size and (pos.min() < 0 or pos.max() >= self.cfg.max_position_embeddings):
            raise ValueError("position out of range of the RoPE table")
        S = ids.shape[0]
        rank = np.arange(S) if rank is None else np.asarray(rank).reshape(-1)
        h = self.w.rows("model.embed_tokens.weight", ids).astype(np.float32)
        new = []
        for l in range(self.cfg.num_hidden_layers):
            c = kv_caches[l] if kv_caches is not None else None
            h, kv = self._layer(l, h, pos, c, rank)
            new.append(kv)
        h = self._r(rms_norm(h, self.w["model.norm.weight"], self.cfg.rms_norm_eps))
        if logits_rows is not None:
            h = h[logits_rows]
        if return_hidden:
            return h, new
        logits = self._lm_head(h)
        if round_logits:
            logits = self._r(logits)
        return logits, new

    def forward(self, input_ids, position_offset: int = 0, kv_caches=None):
        """``WeDLMForCausalLM::forward`` (``causal_lm.rs:46-56``): sequential positions."""
        ids = np.asarray(input_ids, dtype=np.int64).reshape(-1)
        pos = np.arange(position_offset, position_offset + ids.shape[0])
        return self.forward_with_positions(ids, pos, kv_caches)

    def prefill_cache(self, input_ids):
        """K/V of a causal forward over ``input_ids`` at positions ``0..P-1`` without
        the LM head (what ``cache_prefix`` keeps, ``wedlm.rs:85-96``)."""
        ids = np.asarray(input_ids, dtype=np.int64).reshape(-1)
        pos = np.arange(ids.shape[0])
        h = self.w.rows("model.embed_tokens.weight", ids).astype(np.float32)
        new = []
        for l in range(self.cfg.num_hidden_layers):
            h, kv = self._layer(l, h, pos, None, np.arange(ids.shape[0]))
            new.append(kv)
        return new
