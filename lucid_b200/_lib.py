"""ctypes binding of liblucid_b200.so (the C ABI in include/lucid_b200.h).

The shared library is built in-tree by ``python -m lucid_b200.build``.  There
is no fallback: if the library is missing or fails to load, every op raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liblucid_b200.so")

LUCID_OK = 0
KERNEL_IDS = {"prep": 1, "solve_fwd": 2, "attn_fwd": 3, "attn_bwd": 4, "solve_bwd": 5, "attn_bwd_row": 6,
              "solve_bwd_row": 7, "path_block": 8, "path_scores": 9, "path_solve": 10, "path_solve_t": 11,
              "path_row": 12, "path_col": 13, "path_attn": 14, "decode": 15}
ERRORS = {
    1: "unsupported shape (head_dim at most 128, Hq a multiple of Hkv)",
    2: "pointer or stride not 16-byte aligned",
    3: "workspace missing or too small",
    4: "TMA descriptor creation failed",
    5: "CUDA launch error",
    6: "problem exceeds a fixed-size internal buffer",
}

c_int, c_float, c_size_t, c_void_p, c_int64 = (
    ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_int64)
c_float_p = ctypes.POINTER(ctypes.c_float)

S3 = [c_int64] * 3  # (sb, sh, sn) element strides

# name -> (restype, argtypes); every symbol declared in include/lucid_b200.h
SIGNATURES = {
    "lucid_version": (c_int, []),
    "lucid_padded_len": (c_int, [c_int]),
    "lucid_workspace_status_offset": (c_size_t, []),
    "lucid_solve_fwd_workspace_bytes": (c_size_t, [c_int] * 4),
    "lucid_solve_fwd": (c_int, [c_int] * 4 + [c_float, c_float] + [c_void_p] + S3 + [c_void_p] + S3
                        + [c_void_p] * 5 + [c_void_p, c_size_t, c_void_p]),
    "lucid_solve_fwd_noalloc": (c_int, [c_int] * 4 + [c_float, c_float] + [c_void_p] + S3 + [c_void_p] + S3
                                + [c_void_p] * 5 + [c_void_p]),
    "lucid_attn_fwd_workspace_bytes": (c_size_t, [c_int] * 5),
    "lucid_attn_fwd": (c_int, [c_int] * 5 + [c_float] + [c_void_p] + S3 + [c_void_p] + S3 + [c_void_p]
                       + [c_void_p] + S3 + [c_void_p] + [c_void_p, c_size_t, c_void_p]),
    "lucid_attn_bwd_workspace_bytes": (c_size_t, [c_int] * 5),
    "lucid_attn_bwd_fast_workspace_bytes": (c_size_t, [c_int] * 5),
    "lucid_attn_bwd": (c_int, [c_int] * 5 + [c_float] + [c_void_p] + S3 + [c_void_p] + S3 + [c_void_p]
                       + [c_void_p] + S3 + [c_void_p] + S3 + [c_void_p] + [c_void_p] + S3
                       + [c_void_p, c_void_p] + [c_void_p, c_size_t, c_void_p]),
    "lucid_solve_bwd_workspace_bytes": (c_size_t, [c_int] * 4),
    "lucid_solve_bwd_fast_workspace_bytes": (c_size_t, [c_int] * 4),
    "lucid_solve_bwd": (c_int, [c_int] * 4 + [c_float] + [c_void_p] + S3 + [c_void_p] * 5
                        + [c_void_p, c_void_p] + [c_void_p] + S3 + [c_void_p] + S3
                        + [c_void_p, c_size_t, c_void_p]),
    "lucid_path_fwd_workspace_bytes": (c_size_t, [c_int] * 5),
    "lucid_path_fwd": (c_int, [c_int] * 5 + [c_float] + ([c_void_p] + S3) * 4 + [c_void_p, c_int] + S3
                       + [c_void_p] + S3 + [c_void_p] + S3 + [c_void_p, c_size_t, c_void_p]),
    "lucid_path_bwd_workspace_bytes": (c_size_t, [c_int] * 5),
    "lucid_path_bwd": (c_int, [c_int] * 5 + [c_float] + ([c_void_p] + S3) * 3 + [c_void_p, c_int] + S3
                       + [c_void_p] + S3 + [c_void_p, c_size_t] + ([c_void_p] + S3) * 4 + [c_void_p, c_int] + S3
                       + [c_void_p, c_size_t, c_void_p]),
    "lucid_path_attn_fwd_workspace_bytes": (c_size_t, [c_int] * 5),
    "lucid_path_attn_fwd": (c_int, [c_int] * 5 + [c_float] + ([c_void_p] + S3) * 4 + [c_void_p, c_int] + S3
                            + [c_void_p] + S3 + [c_void_p] + S3 + [c_void_p, c_size_t, c_void_p]),
    "lucid_decode_workspace_bytes": (c_size_t, [c_int] * 5),
    "lucid_decode_update": (c_int, [c_int] * 5 + [c_float, c_float] + ([c_void_p] + S3) * 5
                            + [c_void_p, c_size_t, c_void_p]),
    "lucid_decode_attn_workspace_bytes": (c_size_t, [c_int] * 5),
    "lucid_decode_attn": (c_int, [c_int] * 6 + [c_float] + ([c_void_p] + S3) * 4 + [c_void_p, c_size_t, c_void_p]),
    "lucid_decode_step_fused": (c_int, [c_int] * 3),
    "lucid_decode_step_workspace_bytes": (c_size_t, [c_int] * 6),
    "lucid_decode_step": (c_int, [c_int] * 6 + [c_float, c_float] + ([c_void_p] + S3) * 7
                          + [c_void_p, c_size_t, c_void_p]),
    "lucid_cp_prep": (c_int, [c_int] * 4 + [c_float, c_float] + [c_int] * 3 + [c_void_p] + S3
                      + [c_void_p] * 4 + [c_void_p]),
    "lucid_cp_publish": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "lucid_cp_solve_fwd": (c_int, [c_int] * 4 + [c_float, c_int, c_int, c_int] + [c_void_p] + S3
                           + [c_void_p] * 6 + [c_void_p]),
    "lucid_cp_attn_fwd": (c_int, [c_int] * 5 + [c_float, c_int, c_int, c_int] + [c_void_p] + S3 + [c_void_p] + S3
                          + [c_void_p] + [c_void_p] + S3 + [c_void_p, c_void_p, c_void_p]),
    "lucid_cp_delta": (c_int, [c_int] * 6 + [c_void_p] + S3 + [c_void_p] + S3 + [c_void_p, c_void_p]),
    "lucid_cp_attn_bwd": (c_int, [c_int] * 5 + [c_float] + [c_int] * 4 + [c_void_p] + S3 + [c_void_p] + S3
                          + [c_void_p] + [c_void_p] + S3 + [c_void_p] * 2 + [c_void_p] + S3 + [c_void_p] * 4),
    "lucid_cp_solve_bwd": (c_int, [c_int] * 4 + [c_float] + [c_int] * 4 + [c_void_p] + S3 + [c_void_p] * 11
                           + [c_void_p] + S3 + [c_void_p] + S3 + [c_void_p] * 2),
    "lucid_selftest_umma": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "lucid_profile_enable": (c_int, [c_int]),
    "lucid_profile_read": (c_int, [c_float_p, ctypes.POINTER(c_int)]),
}

_lock = threading.Lock()
_lib = None


class LucidError(RuntimeError):
    pass


def load(path: str | None = None):
    """Load (once) and return the ctypes handle of liblucid_b200.so."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise LucidError(
                f"{p} not found: build it with `python -m lucid_b200.build` (no CPU fallback exists)")
        lib = ctypes.CDLL(p)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(rc: int, what: str) -> None:
    if rc != LUCID_OK:
        raise LucidError(f"{what} failed: {ERRORS.get(rc, rc)}")
