"""ctypes binding of libhayate_b200.so (the C ABI in include/hayate_b200.h).

The library is built in-tree (``python -m hayate_b200.build``).  There is no
fallback: if the shared library is missing or fails to load, every kernel
entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libhayate_b200.so")

_lock = threading.Lock()
_lib = None

P = C.c_void_p
I32 = C.c_int32
I64 = C.c_int64
F32 = C.c_float
SZ = C.c_size_t

# name -> (restype, argtypes); mirrors include/hayate_b200.h
SIGNATURES = {
    "hy_version": (C.c_int, []),
    "hy_get_last_error": (C.c_char_p, []),
    "hy_block_pool_init": (C.c_int, [P, P, I32, P]),
    "hy_pack_batch": (C.c_int, [P, I32, I32, P, I32, I32, P, I32, P, P, P, I32, P, P, P, P, P,
                                P, P, P, P]),
    "hy_free_blocks": (C.c_int, [P, I32, I32, P, I32, P, P, P, I32, P, P]),
    "hy_free_blocks_from": (C.c_int, [P, P, I32, I32, P, I32, P, P, P, I32, P, P]),
    "hy_push_blocks": (C.c_int, [P, I32, P, P, I32, P, P]),
    "hy_commit_tokens": (C.c_int, [P, I32, P, P, I32, P, I32, I32, P, P]),
    "hy_qk_norm_rope": (C.c_int, [I32, P, I64, I32, I32, I32, P, P, P, P, P, I32, F32, P, P, P,
                                  P, I32, P, P]),
    "hy_kv_append": (C.c_int, [I32, P, P, I32, I32, P, P, I32, P, P]),
    "hy_attention_workspace_size": (SZ, [I32, I32, I32]),
    "hy_attention_plan": (C.c_int, [P, P, I32, I32, I32, I32, P, SZ, P, P]),
    "hy_varlen_attention": (C.c_int, [I32, P, P, I32, I32, I32, P, I32, I32, I32, P, I32, P, P,
                                      P, I32, F32, I32, I32, P, SZ, I32, P, P]),
    "hy_add_rms_norm": (C.c_int, [I32, P, I64, P, I64, I32, I32, P, F32, P, I64, P]),
    "hy_add_rms_norm_splitk": (C.c_int, [I32, P, I64, P, I32, I64, I64, I32, I32, P, F32, P,
                                         I64, P]),
    "hy_gather_add_rms_norm": (C.c_int, [I32, P, I64, P, I32, P, I64, P, I32, I64, I32, I32, P,
                                         F32, P, I64, P, I64, P, P]),
    "hy_silu_mul": (C.c_int, [I32, P, I64, I32, I32, P, I64, P]),
    "hy_argmax": (C.c_int, [I32, P, I64, I32, I32, P, P]),
    "hy_lm_head_argmax_workspace_size": (I64, []),
    "hy_lm_head_argmax": (C.c_int, [P, I64, I32, P, I64, I32, I32, P, P, P, P]),
    "hy_selftest_wait_timeout": (C.c_int, [P, I32, P, P]),
    "hy_selftest_exp2_poly": (C.c_int, [P, P, I32, P]),
    "hy_varlen_attention_noalloc": (C.c_int, [P, P, I32, I32, I32, P, I32, I32, I32, P, I32, P,
                                              P, P, I32, F32, P, P]),
}


class HayateError(RuntimeError):
    pass


def load() -> C.CDLL:
    """Load the library once; raise if it is absent (no CPU fallback exists)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise HayateError(
                f"{LIB_PATH} is missing: build it with `python -m hayate_b200.build`")
        lib = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def exported_symbols():
    return list(SIGNATURES)


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().hy_get_last_error().decode(errors="replace")
        raise HayateError(f"{what} failed (code {rc}): {msg}")
