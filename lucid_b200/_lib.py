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
              "path_row": 12, "path_col": 13, "path_attn": 14, "decode": 15, "fwd_fused": 16}
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
    "lucid_solve_fwd_fast_workspace_bytes": (c_size_t, [c_int] * 4),
    "lucid_solve_fwd": (c_int, [c_int] * 4 + [c_float, c_float] + [c_void_p] + S3 + [c_void_p] + S3
                        + [c_void_p] * 5 + [c_void_p, c_size_t, c_void_p]),
    "lucid_solve_fwd_noalloc": (c_int, [c_int] * 4 + [c_float, c_float] + [c_void_p] + S3 + [c_void_p] + S3
                                + [c_void_p] * 5 + [c_void_p]),
    "lucid_solve_fwd_noalloc_status": (c_int, [c_void_p, c_void_p]),
    "lucid_fused_fwd_workspace_bytes": (c_size_t, [c_int] * 5),
    "lucid_fused_fwd": (c_int, [c_int] * 5 + [c_float, c_float] + ([c_void_p] + S3) * 3 + [c_void_p] * 3
                        + [c_void_p, c_void_p] + [c_void_p] + S3 + [c_void_p, c_void_p]
                        + [c_void_p, c_size_t, c_void_p]),
    "lucid_attn_fwd_workspace_bytes": (c_size_t, [c_int] * 5),
    "lucid_attn_fwd": (c_int, [c_int] * 5 + [c_float] + [c_void_p] + S3 + [c_void_p] + S3 + [c_void_p]
                       + [c_void_p] + S3 + [c_void_p, c_void_p] + [c_void_p, c_size_t, c_void_p]),
    "lucid_attn_bwd_workspace_bytes": (c_size_t, [c_int] * 5),
    "lucid_attn_bwd_fast_workspace_bytes": (c_size_t, [c_int] * 5),
    "lucid_attn_bwd": (c_int, [c_int] * 5 + [c_float] + [c_void_p] + S3 + [c_void_p] + S3 + [c_void_p]
                       + [c_void_p] + S3 + [c_void_p] + S3 + [c_void_p, c_void_p] + [c_void_p] + S3
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
                          + [c_void_p] + [c_void_p] + S3 + [c_void_p, c_void_p, c_void_p, c_void_p]),
    "lucid_cp_delta": (c_int, [c_int] * 6 + [c_void_p] + S3 + [c_void_p] + S3 + [c_void_p, c_void_p, c_void_p]),
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


# ---------------------------------------------------------------------------
# run-time status words
# ---------------------------------------------------------------------------
# Every kernel bounds its spin waits (mbarriers, cross-CTA flags of the wavefront
# solves) in time; a wait that runs out ends the launch early and records
#   code | barrier << 8 | kernel << 20
# in the int32 status word at lucid_workspace_status_offset() of the call's workspace.
STATUS_CODES = {1: "an mbarrier wait timed out", 2: "a cross-CTA dependency flag never arrived",
                3: "the shared-memory window was not 1024-byte aligned"}
KERNEL_TAGS = {1: "solve forward", 2: "attention forward", 3: "attention backward column pass",
               4: "transposed-solve column pass", 5: "attention backward row pass",
               6: "solve backward row pass", 7: "tensor-core self test", 8: "LUCID-Path block GEMM",
               9: "LUCID-Path score chain", 10: "LUCID-Path solve", 11: "LUCID-Path transposed solve",
               12: "LUCID-Path row pass", 13: "LUCID-Path column pass", 14: "PaTH attention",
               15: "stored-tile row pass"}


def decode_status(word: int) -> str:
    """Human-readable form of a nonzero status word."""
    code, where, tag = word & 0xFF, (word >> 8) & 0xFFF, (word >> 20) & 0xFF
    msg = f"{KERNEL_TAGS.get(tag, f'kernel {tag}')}: {STATUS_CODES.get(code, f'code {code}')}"
    if code == 1:
        msg += f" (barrier at shared offset {where * 8:#x})"
    return msg + f" [status {word:#x}]"


class _StatusWatch:
    """Reads the status words of launched ops back without stalling the stream.

    After an op's launches, ``watch`` queues an asynchronous copy of its status word
    into pinned host memory (stream-ordered after the kernels, so the workspace may be
    freed right away) and an event.  Completed words are inspected at the next op of
    this module (``poll``) or by ``check_status()``, which waits for all of them; a
    nonzero word raises LucidError naming the kernel and the wait that ran out.
    LUCID_B200_SYNC_STATUS=1 makes every op wait for its own word (debugging).
    """

    def __init__(self):
        self.pending = []
        self.lock = threading.Lock()
        self.sync = os.environ.get("LUCID_B200_SYNC_STATUS", "0") not in ("", "0")

    def watch(self, ws, what: str, offset: int = 0) -> None:
        import torch
        if torch.cuda.is_current_stream_capturing():
            return
        host = torch.empty(1, dtype=torch.int32, pin_memory=True)
        word = ws[offset:offset + 4].view(torch.int32)
        host.copy_(word, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        with self.lock:
            self.pending.append((ev, host, what))
        if self.sync:
            self.wait_all()

    def _take(self, block: bool):
        with self.lock:
            done, keep = [], []
            for item in self.pending:
                if block:
                    item[0].synchronize()
                (done if block or item[0].query() else keep).append(item)
            self.pending = keep
        bad = [(what, int(host[0])) for _, host, what in done if int(host[0]) != 0]
        if bad:
            raise LucidError("; ".join(f"{what}: {decode_status(w)}" for what, w in bad))

    def poll(self) -> None:
        if self.pending:
            self._take(False)

    def wait_all(self) -> None:
        self._take(True)


STATUS = _StatusWatch()


def check_status() -> None:
    """Wait for the status words of every op launched so far and raise LucidError if a
    kernel ended a bounded wait early (its results are then not valid)."""
    STATUS.wait_all()
