"""Host-side mirror of the WeDLM-rs decode API over the B200 C ABI.

``Context`` owns one ``wedlm_ctx`` (one GPU).  The class and method names follow the
reference (``WeDLMForCausalLM``, ``WeDLMDecoder``, ``SamplingParams``); every compute
call goes through ``libwedlm_b200.so``.
"""
from ._lib import BF16, F16, F32, WedlmError, lib  # noqa: F401
from .context import Context, SamplingParams, ModelConfig, comm_unique_id  # noqa: F401
