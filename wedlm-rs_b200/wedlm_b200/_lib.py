"""ctypes binding of ``libwedlm_b200.so`` (the C ABI in ``include/wedlm_b200.h``).

The shared library is built in-tree (``make -C wedlm-rs_b200``) and loaded from this
directory.  There is no fallback: importing the binding without the library raises.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libwedlm_b200.so")

WEDLM_OK = 0
STATUS_NAMES = {0: "OK", -1: "INVALID_ARG", -2: "OOM", -3: "CUDA", -4: "TIMEOUT",
                -5: "NOT_FOUND", -6: "IO", -7: "STATE", -8: "UNSUPPORTED"}
F32, BF16, F16 = 0, 1, 2


class WedlmError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"wedlm error {code} ({STATUS_NAMES.get(code, '?')}): {msg}")
        self.code = code


class WedlmConfig(C.Structure):
    _fields_ = [
        ("vocab_size", C.c_int32), ("hidden_size", C.c_int32), ("num_hidden_layers", C.c_int32),
        ("num_attention_heads", C.c_int32), ("num_key_value_heads", C.c_int32),
        ("head_dim", C.c_int32), ("intermediate_size", C.c_int32),
        ("max_position_embeddings", C.c_int32), ("rope_theta", C.c_double),
        ("rms_norm_eps", C.c_double), ("qk_norm", C.c_int32), ("eos_token_id", C.c_int32),
        ("mask_token_id", C.c_int32), ("dtype", C.c_int32), ("max_block_tokens", C.c_int32),
        ("vocab_shard_begin", C.c_int32), ("vocab_shard_end", C.c_int32),
    ]


class WedlmSamplingParams(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float),
                ("entropy_threshold", C.c_float), ("distance_penalty", C.c_float),
                ("max_tokens_per_step", C.c_int32), ("margin_threshold", C.c_float)]


class WedlmBlockStats(C.Structure):
    _fields_ = [("steps", C.c_int64), ("tokens_generated", C.c_int64),
                ("avg_confidence", C.c_float), ("avg_entropy", C.c_float),
                ("max_entropy", C.c_float), ("high_entropy_count", C.c_int64),
                ("block_size_reductions", C.c_int64), ("cache_refreshes", C.c_int64),
                ("prefix_cached", C.c_int32)]


P = C.c_void_p
I32P = C.POINTER(C.c_int32)

_PROTOS = {
    "wedlm_create": (C.c_int, [C.POINTER(WedlmConfig), C.c_int, C.c_int, C.c_int, C.POINTER(P)]),
    "wedlm_destroy": (None, [P]),
    "wedlm_last_error": (C.c_char_p, [P]),
    "wedlm_get_config": (C.c_int, [P, C.POINTER(WedlmConfig)]),
    "wedlm_set_weight": (C.c_int, [P, C.c_char_p, P, C.c_int, C.POINTER(C.c_int64), C.c_int]),
    "wedlm_init_random": (C.c_int, [P, C.c_uint64, C.c_float]),
    "wedlm_get_weight": (C.c_int, [P, C.c_char_p, P, C.c_int64]),
    "wedlm_reset_sequence": (C.c_int, [P, C.c_int]),
    "wedlm_cache_len": (C.c_int, [P, C.c_int, I32P]),
    "wedlm_commit": (C.c_int, [P, C.c_int, C.c_int]),
    "wedlm_truncate": (C.c_int, [P, C.c_int, C.c_int]),
    "wedlm_prefill": (C.c_int, [P, C.c_int, P, C.c_int, P]),
    "wedlm_block_forward": (C.c_int, [P, C.c_int, P, P, P, P, C.c_int, P, P, C.c_int, I32P, P]),
    "wedlm_entropy_select": (C.c_int, [P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                                       C.c_float, C.c_float, C.c_int, P, P, P, P, P, P, P, P, P]),
    "wedlm_entropy_select_noalloc": (C.c_int, [P, P, C.c_int, C.c_int, C.c_int, C.c_int,
                                               C.c_float, C.c_float, C.c_float, C.c_int, P, P,
                                               P, P, P, P, P, P, P]),
    "wedlm_entropy_partials": (C.c_int, [P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                         C.c_float, P, P]),
    "wedlm_entropy_combine": (C.c_int, [P, P, C.c_int, C.c_int, C.c_float, C.c_float, C.c_int,
                                        P, P, P, P, P, P, P, P, P]),
    "wedlm_generate_streaming": (C.c_int, [P, C.c_int, P, C.c_int, C.c_int, C.c_int,
                                           C.POINTER(WedlmSamplingParams), P, I32P,
                                           C.POINTER(WedlmBlockStats), P]),
    "wedlm_generate_streaming_batch": (C.c_int, [P, C.c_int, P, C.c_int, C.c_int, C.c_int,
                                                 C.POINTER(WedlmSamplingParams), P, P, P, P]),
    "wedlm_decode_begin": (C.c_int, [P, C.c_int, P, P, C.c_int, C.c_int, C.c_int,
                                     C.POINTER(WedlmSamplingParams), P]),
    "wedlm_decode_step": (C.c_int, [P, C.c_int, I32P]),
    "wedlm_decode_result": (C.c_int, [P, C.c_int, P, I32P, C.POINTER(WedlmBlockStats)]),
    "wedlm_decode_io_bytes": (C.c_int, [P, C.POINTER(C.c_int64), C.POINTER(C.c_int64),
                                        C.POINTER(C.c_int64)]),
    "wedlm_decode_end": (C.c_int, [P]),
    "wedlm_set_sampling_seed": (C.c_int, [P, C.c_uint64]),
    "wedlm_kernel_sample": (C.c_int, [P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                                      C.c_float, P, P, P]),
    "wedlm_comm_unique_id": (C.c_int, [P, C.c_int]),
    "wedlm_comm_init": (C.c_int, [P, P, C.c_int, C.c_int, C.c_int]),
    "wedlm_comm_destroy": (C.c_int, [P]),
    # kernel-level entry points (include/wedlm_b200_kernels.h)
    "wedlm_kernel_gemm": (C.c_int, [P, P, C.c_int64, P, P, C.c_int64, C.c_int, C.c_int, C.c_int,
                                    C.c_int, C.c_int, C.c_int, P, C.c_int64, P, C.c_int64, P]),
    "wedlm_kernel_pack_weight": (C.c_int, [P, P, C.c_int64, C.c_int, C.c_int, P, P]),
    "wedlm_check_device_error": (C.c_int, [P, P]),
    "wedlm_kernel_wait_probe": (C.c_int, [P, C.c_int64, P, P]),
    "wedlm_load_weights": (C.c_int, [P, C.c_char_p]),
    "wedlm_generate_block": (C.c_int, [P, C.c_int, P, C.c_int, C.c_int,
                                       C.POINTER(WedlmSamplingParams), P,
                                       C.POINTER(WedlmBlockStats), P]),
    "wedlm_commit_block": (C.c_int, [P, C.c_int, P, C.c_int, P]),
    "wedlm_generate_autoregressive": (C.c_int, [P, C.c_int, P, C.c_int, C.c_int, P, I32P, P]),
    "wedlm_generate_with_stats": (C.c_int, [P, C.c_int, P, C.c_int, C.c_int, C.c_int,
                                            C.POINTER(WedlmSamplingParams), P, I32P,
                                            C.POINTER(WedlmBlockStats), P]),
    "wedlm_kernel_attention_prepare": (C.c_int, [P, P, P, P, C.c_int, C.c_int, C.c_int,
                                                 C.c_int, P, P]),
    "wedlm_kernel_attention_run": (C.c_int, [P, P, P]),
    "wedlm_profile_enable": (C.c_int, [P, C.c_int]),
    "wedlm_profile_read": (C.c_int, [P, C.c_int, C.POINTER(C.c_double), C.POINTER(C.c_double),
                                     C.POINTER(C.c_double), C.POINTER(C.c_int64)]),
    "wedlm_launch_count": (C.c_int, [P, C.POINTER(C.c_int64)]),
}

_lib = None


def lib() -> C.CDLL:
    """Load (once) and return the library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `make -C wedlm-rs_b200` "
                              "(there is no CPU fallback)")
        l = C.CDLL(LIB_PATH)
        for name, (res, args) in _PROTOS.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def check(rc: int, ctx=None) -> None:
    if rc != WEDLM_OK:
        msg = lib().wedlm_last_error(ctx)
        raise WedlmError(rc, msg.decode() if msg else "")


def ptr(t) -> C.c_void_p:
    """Device (or host) address of a torch tensor / numpy array, or NULL."""
    if t is None:
        return None
    if hasattr(t, "data_ptr"):
        return C.c_void_p(t.data_ptr())
    return C.c_void_p(t.ctypes.data)


def stream_ptr(stream=None) -> C.c_void_p:
    import torch
    if stream == 0:
        return None
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)
