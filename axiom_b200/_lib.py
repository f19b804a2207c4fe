"""ctypes binding of ``libkda_b200.so`` (the C ABI declared in ``include/kda_b200.h`` and
``include/kda_mixer.h``).

There is no fallback: if the library is missing or cannot be loaded, every
entry point raises ``RuntimeError``.  Build it with ``python -m axiom_b200.build``.
"""

from __future__ import annotations

import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libkda_b200.so")

KDA_F32 = 0
KDA_BF16 = 1

_P = ctypes.c_void_p
_I = ctypes.c_int
_Z = ctypes.c_size_t
_F = ctypes.c_float

#: every symbol the header declares, with its ctypes signature
SIGNATURES = {
    "kda_version": ([], _I),
    "kda_strerror": ([_I], ctypes.c_char_p),
    "kda_ckpt_bytes": ([_I] * 8, _Z),
    "kda_fwd": ([_P] * 9 + [_I] * 9 + [_P], _I),
    "kda_bwd_workspace_bytes": ([_I] * 7, _Z),
    "kda_bwd": ([_P] * 14 + [_P, _Z] + [_I] * 9 + [_P], _I),
    "kda_decode": ([_P] * 7 + [_I] * 5 + [_P], _I),
    "kda_bwd_noalloc": ([_P] * 14 + [_I] * 9 + [_P], _I),
    "kda_fwd_varlen": ([_P] * 10 + [_I] * 9 + [_P], _I),
    "kda_bwd_varlen_workspace_bytes": ([_I] * 7, _Z),
    "kda_bwd_varlen": ([_P] * 15 + [_Z, _P] + [_I] * 9 + [_P], _I),
    # include/kda_mixer.h
    "kda_prologue_fwd": ([_P] * 10 + [_F, _I] + [_P] * 3 + [_I] + [_P] * 6 + [_I] * 8 + [_P], _I),
    "kda_prologue_bwd_workspace_bytes": ([_I] * 6, _Z),
    "kda_prologue_bwd": ([_P] * 10 + [_F, _I, _P, _P, _I] + [_P] * 18 + [_Z] + [_I] * 8 + [_P], _I),
    "kda_gated_rmsnorm_fwd": ([_P] * 5 + [_I] * 4 + [_F] + [_I] * 3 + [_P], _I),
    "kda_gated_rmsnorm_bwd": ([_P] * 7 + [_I] * 4 + [_F] + [_I] * 3 + [_P], _I),
    "kda_decode_fused": ([_P] * 13 + [_F, _I, _F, _P] + [_I] * 7 + [_P], _I),
    "kda_device_status": ([_P, _I, _P], _I),
    "kda_selftest_wait_timeout": ([ctypes.c_uint, _P], _I),
}

_lib = None


class KDAError(RuntimeError):
    """A non-zero status from the C ABI (``KDA_ERR_*``)."""

    def __init__(self, fn: str, status: int, text: str):
        super().__init__(f"{fn} failed with status {status}: {text}")
        self.status = status


def lib() -> ctypes.CDLL:
    """Load the library once; raise if it is absent (no silent fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"libkda_b200.so is not built ({LIB_PATH}); run `python -m axiom_b200.build`. "
                "There is no CPU or eager fallback for the KDA kernels.")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = res
        _lib = handle
    return _lib


def check(fn: str, status: int) -> None:
    if status != 0:
        text = lib().kda_strerror(status).decode()
        raise KDAError(fn, status, text)
