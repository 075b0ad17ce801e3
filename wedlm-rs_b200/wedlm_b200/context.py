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

    def entropy_select_noalloc(self, logits, temperature: float, tau: float, lam: float,
                               seq_rows, mask_pos, caps, out: dict, stream=None) -> dict:
        """``entropy_select`` through the allocation-free entry point: the caller passes
        the preallocated outputs ``out`` (keys H, argmax, maxprob, selected,
        n_selected) and the kernels use a fixed static device scratch."""
        import torch
        rows, V = logits.shape[0], logits.shape[1]
        dt = BF16 if logits.dtype == torch.bfloat16 else F32
        assert logits.dtype in (torch.bfloat16, torch.float32) and logits.stride(1) == 1
        nseq = seq_rows.numel() - 1
        rc = lib().wedlm_entropy_select_noalloc(
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

    def sample(self, logits, temperature: float, top_p: float, u, out=None, stream=None):
        """T > 0 draw of every row of ``logits`` (CUDA ``[rows, V]``) with the uniforms
        ``u`` (CUDA f32 ``[rows]``): multinomial, or nucleus when ``top_p < 1``."""
        import torch
        rows, V = logits.shape[0], logits.shape[1]
        dt = BF16 if logits.dtype == torch.bfloat16 else F32
        if out is None:
            out = torch.empty(rows, dtype=torch.int32, device=logits.device)
        check(lib().wedlm_kernel_sample(self.h, ptr(logits), dt, rows, V, logits.stride(0),
                                        temperature, top_p, ptr(u), ptr(out), stream_ptr(stream)),
              self.h)
        return out

    def set_sampling_seed(self, seed: int) -> None:
        """Seed of the T > 0 draws of the decode loops."""
        check(lib().wedlm_set_sampling_seed(self.h, seed & ((1 << 64) - 1)), self.h)

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

    # ---- kernel-level entry points ------------------------------------------------------
    EPI_STORE, EPI_STORE_F32, EPI_RESIDUAL, EPI_SWIGLU = 0, 1, 2, 3

    def gemm(self, X, W, out, epilogue: int = 0, W2=None, resid=None, stream=None, N=None):
        """``out[m, n] (epilogue)= sum_k X[m, k] W[n, k]`` through ``wedlm_kernel_gemm``.
        ``W`` is a row-major [N, K] tensor, or a 1-D packed tensor from ``pack_weight``
        (then pass ``N``)."""
        import torch
        M, K = X.shape
        packed = W.dim() == 1
        if not packed:
            N = W.shape[0]
        dt = BF16 if X.dtype == torch.bfloat16 else F32
        rc = lib().wedlm_kernel_gemm(self.h, ptr(X), X.stride(0), ptr(W), ptr(W2),
                                     K if packed else W.stride(0), 1 if packed else 0, M, N, K,
                                     dt, epilogue, ptr(out), out.stride(0), ptr(resid),
                                     resid.stride(0) if resid is not None else 0,
                                     stream_ptr(stream))
        check(rc, self.h)
        return out

    def pack_weight(self, W, stream=None):
        """Packed GEMM tiles of a row-major bf16 [N, K] weight (1-D tensor)."""
        import torch
        N, K = W.shape
        P = torch.zeros(((N + 127) // 128) * 128 * K, dtype=torch.bfloat16, device=W.device)
        check(lib().wedlm_kernel_pack_weight(self.h, ptr(W), W.stride(0), N, K, ptr(P),
                                             stream_ptr(stream)), self.h)
        return P

    def attention_prepare(self, q, k, v, L: int, rank=None, stream=None) -> None:
        """Stand-alone block attention inputs: ``q`` bf16 CUDA ``[S, nh, 128]``, ``k`` /
        ``v`` bf16 CUDA ``[L + S, nkv, 128]`` (cached tokens first), ``rank`` int32 CUDA
        ``[S]`` or None (window index)."""
        S, nh = q.shape[0], q.shape[1]
        nkv = k.shape[1]
        assert q.is_contiguous() and k.is_contiguous() and v.is_contiguous()
        assert k.shape[0] == L + S and v.shape == k.shape and q.shape[2] == 128
        self._att_shape = (S, nh)
        check(lib().wedlm_kernel_attention_prepare(self.h, ptr(q), ptr(k), ptr(v), L, S, nh, nkv,
                                                   ptr(rank) if rank is not None else None,
                                                   stream_ptr(stream)), self.h)

    def attention_run(self, out=None, stream=None):
        """Block attention on the prepared inputs; returns bf16 ``[S, nh * 128]``."""
        import torch
        S, nh = self._att_shape
        if out is None:
            out = torch.empty(S, nh * 128, dtype=torch.bfloat16, device="cuda")
        check(lib().wedlm_kernel_attention_run(self.h, ptr(out), stream_ptr(stream)), self.h)
        return out

    def check_device_error(self, stream=None):
        check(lib().wedlm_check_device_error(self.h, stream_ptr(stream)), self.h)

    def wait_probe(self, limit_ns: int, stream=None):
        """Launch the bounded-wait probe (a wait that nothing completes); returns the
        device int32 tensor {wait succeeded, microseconds waited}."""
        import torch
        out = torch.full((2,), -1, dtype=torch.int32, device=f"cuda:{self.device}")
        check(lib().wedlm_kernel_wait_probe(self.h, int(limit_ns), ptr(out), stream_ptr(stream)),
              self.h)
        return out

    # ---- model: weights ---------------------------------------------------------------
    def load_safetensors(self, model_dir: str) -> None:
        """All model tensors from ``model_dir`` (model.safetensors, or the shards of
        model.safetensors.index.json)."""
        check(lib().wedlm_load_weights(self.h, str(model_dir).encode()), self.h)

    def set_weight(self, name: str, array) -> None:
        """Upload one checkpoint tensor (numpy f32 / f16, or uint16 bf16 bit patterns
        with ``bf16=True`` semantics via dtype uint16)."""
        import numpy as np
        a = np.ascontiguousarray(array)
        if a.dtype == np.float32:
            dt = F32
        elif a.dtype == np.float16:
            dt = 2
        elif a.dtype == np.uint16:
            dt = BF16
        else:
            a = np.ascontiguousarray(a, dtype=np.float32)
            dt = F32
        shape = (C.c_int64 * a.ndim)(*a.shape)
        check(lib().wedlm_set_weight(self.h, name.encode(), a.ctypes.data, dt, shape, a.ndim),
              self.h)

    def load_weights(self, weights: dict) -> None:
        for k, v in weights.items():
            self.set_weight(k, v)

    def init_random(self, seed: int = 0, std: float = 0.02) -> None:
        check(lib().wedlm_init_random(self.h, seed, std), self.h)

    def get_weight(self, name: str, shape):
        """Stored tensor in the model dtype (bf16 returned as uint16 bit patterns;
        norm weights as f32)."""
        import numpy as np
        is_norm = name.endswith("norm.weight")
        dt = np.float32 if (is_norm or self.config.dtype_code == F32) else np.uint16
        out = np.empty(shape, dtype=dt)
        check(lib().wedlm_get_weight(self.h, name.encode(), out.ctypes.data, out.nbytes), self.h)
        return out

    # ---- model: KV cache ----------------------------------------------------------------
    def reset_sequence(self, seq: int = 0) -> None:
        check(lib().wedlm_reset_sequence(self.h, seq), self.h)

    def cache_len(self, seq: int = 0) -> int:
        v = C.c_int32()
        check(lib().wedlm_cache_len(self.h, seq, C.byref(v)), self.h)
        return v.value

    def commit(self, seq: int, n_commit: int) -> None:
        check(lib().wedlm_commit(self.h, seq, n_commit), self.h)

    def truncate(self, seq: int, new_len: int) -> None:
        check(lib().wedlm_truncate(self.h, seq, new_len), self.h)

    def prefill(self, seq: int, ids, stream=None) -> None:
        import numpy as np
        a = np.ascontiguousarray(ids, dtype=np.int32)
        check(lib().wedlm_prefill(self.h, seq, a.ctypes.data, a.size, stream_ptr(stream)),
              self.h)

    # ---- model: forward -------------------------------------------------------------------
    def forward_with_positions(self, seqs, tokens, positions, rank=None, logit_row_begin=None,
                               logits_dtype=None, stream=None):
        """``WeDLMForCausalLM::forward_with_positions`` for ``len(seqs)`` windows of equal
        length S (``tokens`` / ``positions`` / ``rank``: int arrays ``[nseq, S]``).
        Returns the logits of rows ``logit_row_begin[b]:S`` of every window, packed, as a
        CUDA tensor (model dtype unless ``logits_dtype`` is torch.float32)."""
        import numpy as np
        import torch
        seqs = np.ascontiguousarray(np.atleast_1d(seqs), dtype=np.int32)
        tok = np.ascontiguousarray(np.atleast_2d(tokens), dtype=np.int32)
        pos = np.ascontiguousarray(np.atleast_2d(positions), dtype=np.int32)
        nseq, S = tok.shape
        rk = None if rank is None else np.ascontiguousarray(np.atleast_2d(rank), dtype=np.int32)
        lb = np.zeros(nseq, np.int32) if logit_row_begin is None else \
            np.ascontiguousarray(np.atleast_1d(logit_row_begin), dtype=np.int32)
        nrows = int(sum(S - int(b) for b in lb))
        V = (self.config.vocab_shard_end - self.config.vocab_shard_begin) or self.config.vocab_size
        model_dt = torch.float32 if self.config.dtype_code == F32 else torch.bfloat16
        tdt = logits_dtype or model_dt
        logits = torch.empty(max(nrows, 1), V, dtype=tdt, device=f"cuda:{self.device}")
        n = C.c_int32()
        check(lib().wedlm_block_forward(self.h, nseq, seqs.ctypes.data, tok.ctypes.data,
                                        pos.ctypes.data, rk.ctypes.data if rk is not None else None,
                                        S, lb.ctypes.data, ptr(logits),
                                        F32 if tdt == torch.float32 else BF16, C.byref(n),
                                        stream_ptr(stream)), self.h)
        return logits[:n.value]

    # ---- decode loops ---------------------------------------------------------------------
    def generate_streaming(self, prompt, max_new_tokens: int, window_size: int,
                           params: SamplingParams, seq: int = 0, stream=None):
        """``WeDLMDecoder::generate_streaming``: returns (prompt + generated ids, stats)."""
        import numpy as np
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(max_new_tokens, 1), np.int32)
        n = C.c_int32()
        st = WedlmBlockStats()
        pc = params.to_c()
        check(lib().wedlm_generate_streaming(self.h, seq, p.ctypes.data, p.size, max_new_tokens,
                                             window_size, C.byref(pc), out.ctypes.data,
                                             C.byref(n), C.byref(st), stream_ptr(stream)), self.h)
        stats = {f: getattr(st, f) for f, _ in WedlmBlockStats._fields_}
        return list(p) + out[:n.value].tolist(), stats

    def generate_block(self, prefix, block_size: int, params: SamplingParams, seq: int = 0,
                       stream=None):
        """``WeDLMDecoder::generate_block``: returns (prefix + block, block, stats)."""
        import numpy as np
        p = np.ascontiguousarray(prefix, dtype=np.int32)
        out = np.zeros(block_size, np.int32)
        st = WedlmBlockStats()
        pc = params.to_c()
        check(lib().wedlm_generate_block(self.h, seq, p.ctypes.data, p.size, block_size,
                                         C.byref(pc), out.ctypes.data, C.byref(st),
                                         stream_ptr(stream)), self.h)
        stats = {f: getattr(st, f) for f, _ in WedlmBlockStats._fields_}
        return list(p) + out.tolist(), out.tolist(), stats

    def generate_autoregressive(self, prompt, max_new_tokens: int, seq: int = 0, stream=None):
        """``WeDLMEngine::generate_autoregressive`` at T = 0: returns the generated ids."""
        import numpy as np
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(max_new_tokens, 1), np.int32)
        n = C.c_int32()
        check(lib().wedlm_generate_autoregressive(self.h, seq, p.ctypes.data, p.size,
                                                  max_new_tokens, out.ctypes.data, C.byref(n),
                                                  stream_ptr(stream)), self.h)
        return out[:n.value].tolist()

    def commit_block(self, block, seq: int = 0, stream=None) -> None:
        """``WeDLMDecoder::commit_block_to_cache``."""
        import numpy as np
        b = np.ascontiguousarray(block, dtype=np.int32)
        check(lib().wedlm_commit_block(self.h, seq, b.ctypes.data, b.size, stream_ptr(stream)),
              self.h)

    def generate_with_stats(self, prompt, max_new_tokens: int, block_size: int,
                            params: SamplingParams, seq: int = 0, stream=None):
        """``WeDLMDecoder::generate_with_stats``: returns (prompt + blocks, stats)."""
        import numpy as np
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(p.size + max_new_tokens + block_size, np.int32)
        n = C.c_int32()
        st = WedlmBlockStats()
        pc = params.to_c()
        check(lib().wedlm_generate_with_stats(self.h, seq, p.ctypes.data, p.size, max_new_tokens,
                                              block_size, C.byref(pc), out.ctypes.data,
                                              C.byref(n), C.byref(st), stream_ptr(stream)), self.h)
        stats = {f: getattr(st, f) for f, _ in WedlmBlockStats._fields_}
        return out[:n.value].tolist(), stats

    def generate_streaming_batch(self, prompts, max_new_tokens: int, window_size: int,
                                 params: SamplingParams, stream=None):
        import numpy as np
        p = np.ascontiguousarray(prompts, dtype=np.int32)
        nseq, P = p.shape
        out = np.zeros((nseq, max(max_new_tokens, 1)), np.int32)
        n = np.zeros(nseq, np.int32)
        steps = np.zeros(nseq, np.int64)
        pc = params.to_c()
        check(lib().wedlm_generate_streaming_batch(self.h, nseq, p.ctypes.data, P, max_new_tokens,
                                                   window_size, C.byref(pc), out.ctypes.data,
                                                   n.ctypes.data, steps.ctypes.data,
                                                   stream_ptr(stream)), self.h)
        return [out[b, :n[b]].tolist() for b in range(nseq)], steps

    # ---- step-wise streaming decode session ----------------------------------------------
    def comm_init(self, unique_id: bytes, rank: int, nranks: int, timeout_ms: int = 30000) -> None:
        """Join an NCCL communicator (collective over ``nranks`` processes, one GPU
        each).  The ranks' vocab shards must tile [0, V) in rank order; the decode loops
        then run the LM head and the entropy pass vocabulary-sharded."""
        buf = C.create_string_buffer(bytes(unique_id), 128)
        check(lib().wedlm_comm_init(self.h, buf, rank, nranks, timeout_ms), self.h)

    def comm_destroy(self) -> None:
        check(lib().wedlm_comm_destroy(self.h), self.h)

    def decode_begin(self, seq_ids, prompts, max_new_tokens: int, window_size: int,
                     params: SamplingParams, stream=None) -> None:
        import numpy as np
        sid = np.ascontiguousarray(np.atleast_1d(seq_ids), dtype=np.int32)
        p = np.ascontiguousarray(np.atleast_2d(prompts), dtype=np.int32)
        self._decode_max_new = max_new_tokens
        pc = params.to_c()
        check(lib().wedlm_decode_begin(self.h, sid.size, sid.ctypes.data, p.ctypes.data,
                                       p.shape[1], max_new_tokens, window_size, C.byref(pc),
                                       stream_ptr(stream)), self.h)

    def decode_step(self, n_steps: int = 1) -> int:
        live = C.c_int32()
        check(lib().wedlm_decode_step(self.h, n_steps, C.byref(live)), self.h)
        return live.value

    def decode_result(self, b: int = 0):
        import numpy as np
        out = np.zeros(max(self._decode_max_new, 1), np.int32)
        n = C.c_int32()
        st = WedlmBlockStats()
        check(lib().wedlm_decode_result(self.h, b, out.ctypes.data, C.byref(n), C.byref(st)),
              self.h)
        return out[:n.value].tolist(), {f: getattr(st, f) for f, _ in WedlmBlockStats._fields_}

    def decode_io_bytes(self):
        s, a, b = C.c_int64(), C.c_int64(), C.c_int64()
        check(lib().wedlm_decode_io_bytes(self.h, C.byref(s), C.byref(a), C.byref(b)), self.h)
        return s.value, a.value, b.value

    def decode_end(self) -> None:
        check(lib().wedlm_decode_end(self.h), self.h)

    # ---- profiling --------------------------------------------------------------------------
    KERNEL_CLASSES = ("gemm", "attention", "entropy", "other", "comm")

    def profile_enable(self, on: bool = True) -> None:
        check(lib().wedlm_profile_enable(self.h, 1 if on else 0), self.h)

    def profile_read(self) -> dict:
        out = {}
        for i, name in enumerate(self.KERNEL_CLASSES):
            ms, by, fl, n = C.c_double(), C.c_double(), C.c_double(), C.c_int64()
            check(lib().wedlm_profile_read(self.h, i, C.byref(ms), C.byref(by), C.byref(fl),
                                           C.byref(n)), self.h)
            out[name] = {"ms": ms.value, "bytes": by.value, "flops": fl.value,
                         "launches": n.value}
        return out

    def launch_count(self) -> int:
        v = C.c_int64()
        check(lib().wedlm_launch_count(self.h, C.byref(v)), self.h)
        return v.value


def comm_unique_id() -> bytes:
    """A fresh 128-byte NCCL unique id (make it on one rank, hand it to every rank)."""
    buf = C.create_string_buffer(128)
    check(lib().wedlm_comm_unique_id(buf, 128))
    return buf.raw
