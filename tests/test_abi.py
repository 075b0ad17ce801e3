"""The C-ABI library loads and exports every entry point ``include/wedlm_b200.h``
declares (no compute calls: this runs without a GPU)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", h) for h in ("wedlm_b200.h", "wedlm_b200_kernels.h")]


def header_symbols():
    syms = set()
    for h in HEADERS:
        txt = open(h).read()
        syms |= set(re.findall(r"^WEDLM_API\s+[\w\s\*]*?\b(wedlm_\w+)\s*\(", txt, re.M))
    return sorted(syms)


def test_header_declares_entry_points():
    syms = header_symbols()
    assert "wedlm_create" in syms and "wedlm_entropy_select" in syms
    assert len(syms) >= 18


def test_library_exports_every_declared_symbol():
    from wedlm_b200 import _lib
    l = _lib.lib()
    missing = [s for s in header_symbols() if not hasattr(l, s)]
    assert not missing, missing
    # every declared symbol has a Python prototype
    assert set(header_symbols()) <= set(_lib._PROTOS)


def test_create_without_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from wedlm_b200 import Context, WedlmError
    with pytest.raises(WedlmError) as e:
        Context(None)
    assert e.value.code in (-3, -8)


def test_config_struct_layout():
    from wedlm_b200._lib import WedlmConfig
    from wedlm_b200 import ModelConfig
    c = ModelConfig.wedlm_8b().to_c()
    assert c.vocab_size == 151936 and c.num_key_value_heads == 8 and c.dtype == 1
    # layout: 8 int32, 2 double, 7 int32 (with padding after the first 8 ints: none)
    assert ctypes.sizeof(WedlmConfig) == 8 * 4 + 2 * 8 + 7 * 4 + 4


def test_comm_unique_id_without_gpu():
    """The NCCL unique id needs no device (NCCL is loaded at run time by the library)."""
    from wedlm_b200 import comm_unique_id
    a, b = comm_unique_id(), comm_unique_id()
    assert len(a) == 128 and len(b) == 128 and a != b
