"""``Context``: one ``wedlm_ctx`` (model, KV cache, scratch) on one GPU."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, asdict, field
from typing import Optional, Sequence

from ._lib import (BF16, F32, WedlmBlockStats, WedlmConfig, WedlmSamplingParams, check, lib,
                   ptr, stream_ptr)


@dataclass
class SamplingParams:
    """``SamplingParams`` (reference ``src/decoding/sampler.rs:12-44``)."""

    temperature: float = 0.2
    top_p: float = 1.0
    entropy_threshold: float = 0.6
    distance_penalty: float = 0.02
    max_tokens_per_step: int = 4
    margin_threshold: float = 0.0

    @staticmethod
    def preset(name: str, temperature: float = 0.0) -> "SamplingParams":
        """``Preset::to_params`` (reference ``src/bin/cli.rs:113-137``)."""
        tau, lam, cap = {"quality": (0.5, 0.10, 4), "balanced": (0.8, 0.05, 8),
                         "fast": (1.0, 0.05, 6)}[name]
        return SamplingParams(temperature=temperature, entropy_threshold=tau,
                              distance_penalty=lam, max_tokens_per_step=cap)

    def to_c(self) -> WedlmSamplingParams:
        return WedlmSamplingParams(self.temperature, self.top_p, self.entropy_threshold,
                                   self.distance_penalty, self.max_tokens_per_step,
                                   self.margin_threshold)


@dataclass
class ModelConfig:
    """Shape fields of ``WeDLMConfig`` (reference ``src/config.rs:9-78``)."""

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
    mask_token_id: int = 151665
    dtype: str = "bfloat16"
    max_block_tokens: int = 128
    vocab_shard_begin: int = 0
    vocab_shard_end: int = 0

    @staticmethod
    def wedlm_8b(**kw) -> "ModelConfig":
        """``WeDLMConfig::wedlm_8b`` (reference ``src/config.rs:127-150``); the decoder's
        mask id is ``MASK_TOKEN_ID = 151665`` (``src/lib.rs:20``)."""
        c = ModelConfig(vocab_size=151936, hidden_size=4096, num_hidden_layers=36,
                        num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                        intermediate_size=12288, eos_token_id=151643, mask_token_id=151665)
        for k, v in kw.items():
            setattr(c, k, v)
        return c

    @staticmethod
    def from_dict(d: dict) -> "ModelConfig":
        keys = ModelConfig.__dataclass_fields__.keys()
        c = ModelConfig(**{k: d[k] for k in keys if k in d and d[k] is not None})
        return c

    @property
    def dtype_code(self) -> int:
        return F32 if self.dtype.lower() in ("float32", "f32") else BF16

    def to_c(self) -> WedlmConfig:
        return WedlmConfig(self.vocab_size, self.hidden_size, self.num_hidden_layers,
                           self.num_attention_heads, self.num_key_value_heads, self.head_dim,
                           self.intermediate_size, self.max_position_embeddings,
                           float(self.rope_theta), float(self.rms_norm_eps), int(self.qk_norm),
                           self.eos_token_id, self.mask_token_id, self.dtype_code,
                           self.max_block_tokens, self.vocab_shard_begin, self.vocab_shard_end)


class Context:
    """Owns a ``wedlm_ctx``.  ``config=None`` makes a kernel-only context (the
    entropy-select entry points need no model)."""

    def __init__(self, config: Optional[ModelConfig] = None, device: int = 0, max_seqs: int = 1,
                 max_ctx: int = 4096):
        self.config = config
        self.device = device
        h = C.c_void_p()
        cc = config.to_c() if config is not None else None
        rc = lib().wedlm_create(C.byref(cc) if cc is not None else None, device, max_seqs,
                                max_ctx, C.byref(h))
        check(rc, None)
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().wedlm_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # ---- fused entropy-select ---------------------------------------------------------
    def entropy_select(self, logits, temperature: float, tau: float, lam: float, seq_rows,
                       mask_pos, caps, out: Optional[dict] = None, stream=None) -> dict:
        """One pass over ``logits`` (CUDA tensor ``[rows, >= V]``): entropy, argmax,
        max-prob per row and the commit selection per sequence.  ``seq_rows``,
        ``mask_pos``, ``caps`` are int32 CUDA tensors."""
        import torch
        rows, V = logits.shape[0], logits.shape[1]
        dt = BF16 if logits.dtype == torch.bfloat16 else F32
        assert logits.dtype in (torch.bfloat16, torch.float32) and logits.stride(1) == 1
        nseq = seq_rows.numel() - 1
        dev = logits.device
        if out is None:
            out = {"H": torch.empty(rows, dtype=torch.float32, device=dev),
                   "argmax": torch.empty(rows, dtype=torch.int32, device=dev),
                   "maxprob": torch.empty(rows, dtype=torch.float32, device=dev),
                   "selected": torch.empty(max(rows, 1), dtype=torch.int32, device=dev),
                   "n_selected": torch.empty(nseq, dtype=torch.int32, device=dev)}
        rc = lib().wedlm_entropy_select(
            self.h, ptr(logits), dt, rows, V, logits.stride(0), temperature, tau, lam, nseq,
            ptr(seq_rows), ptr(mask_pos), ptr(caps), ptr(out["H"]), ptr(out["argmax"]),
            ptr(out["maxprob"]), ptr(out["selected"]), ptr(out["n_selected"]), stream_ptr(stream))
        check(rc, self.h)
        return out

    def entropy_partials(self, logits, vocab_offset: int, temperature: float, out=None,
                         stream=None):
        import torch
        rows, V = logits.shape[0], logits.shape[1]
        dt = BF16 if logits.dtype == torch.bfloat16 else F32
        if out is None:
            out = torch.empty(rows, 4, dtype=torch.float32, device=logits.device)
        rc = lib().wedlm_entropy_partials(self.h, ptr(logits), dt, rows, V, logits.stride(0),
                                          vocab_offset, temperature, ptr(out), stream_ptr(stream))
        check(rc, self.h)
        return out

    def entropy_combine(self, partials, tau: float, lam: float, seq_rows, mask_pos, caps,
                        stream=None) -> dict:
        """``partials``: CUDA f32 ``[nshards, rows, 4]``."""
        import torch
        nshards, rows = partials.shape[0], partials.shape[1]
        nseq = seq_rows.numel() - 1
        dev = partials.device
        out = {"H": torch.empty(rows, dtype=torch.float32, device=dev),
               "argmax": torch.empty(rows, dtype=torch.int32, device=dev),
               "maxprob": torch.empty(rows, dtype=torch.float32, device=dev),
               "selected": torch.empty(max(rows, 1), dtype=torch.int32, device=dev),
               "n_selected": torch.empty(nseq, dtype=torch.int32, device=dev)}
        rc = lib().wedlm_entropy_combine(self.h, ptr(partials), nshards, rows, tau, lam, nseq,
                                         ptr(seq_rows), ptr(mask_pos), ptr(caps), ptr(out["H"]),
                                         ptr(out["argmax"]), ptr(out["maxprob"]),
                                         ptr(out["selected"]), ptr(out["n_selected"]),
                                         stream_ptr(stream))
        check(rc, self.h)
        return out
