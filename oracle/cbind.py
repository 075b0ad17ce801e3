"""ctypes binding of the C restatement ``oracle/entropy_ref.c`` (test infrastructure
only: the checker and the timed CPU baseline)."""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "liboracle_entropy.so")
_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_SO):
            build()
        l = C.CDLL(_SO)
        P = C.c_void_p
        l.oracle_entropy_select.restype = C.c_int
        l.oracle_entropy_select.argtypes = [P, C.c_int, C.c_int, C.c_int, C.c_long, C.c_float,
                                            C.c_float, C.c_float, C.c_int, P, P, P, P, P, P, P,
                                            C.c_int]
        _lib = l
    return _lib


def entropy_select(logits: np.ndarray, dtype: str, T: float, tau: float, lam: float,
                   seq_rows, mask_pos, caps, nthreads: int = 0, V: int | None = None):
    """``logits``: float32 array, or uint16 bf16 bit patterns when dtype == 'bf16'."""
    rows, ld = logits.shape
    V = ld if V is None else V
    seq_rows = np.ascontiguousarray(seq_rows, np.int32)
    mask_pos = np.ascontiguousarray(mask_pos, np.int32)
    caps = np.ascontiguousarray(caps, np.int32)
    nseq = len(seq_rows) - 1
    H = np.zeros(rows, np.float32)
    tok = np.zeros(rows, np.int32)
    sel = np.zeros(max(rows, 1), np.int32)
    nsel = np.zeros(nseq, np.int32)
    x = np.ascontiguousarray(logits)
    lib().oracle_entropy_select(x.ctypes.data, 0 if dtype == "f32" else 1, rows, V, ld, T, tau,
                                lam, nseq, seq_rows.ctypes.data, mask_pos.ctypes.data,
                                caps.ctypes.data, H.ctypes.data, tok.ctypes.data, sel.ctypes.data,
                                nsel.ctypes.data, nthreads)
    return {"H": H, "tokens": tok, "selected": sel, "n_selected": nsel}
