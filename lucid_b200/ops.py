"""Torch-facing LUCID ops on the B200 kernels.

Stages (each a thin wrapper over one C-ABI entry point, see
include/lucid_b200.h):

  solve_fwd   X = P^-1 V                      modeling_lucid.py:551-574
  attn_fwd    O = softmax(s Q K^T + causal) X  modeling_lucid.py:505-549
  attn_bwd    dQ, dK(attention), dX
  solve_bwd   dV = P^-T dX, dK through P and RMSNorm  modeling_lucid.py:314-382

Autograd functions:

  LucidSolveFunction      drop-in for get_v_prime's "exp_k_norm" branch
  LucidAttnFunction       drop-in for eager_lucid_attention_forward
  LucidAttentionFunction  the fused op (solve + attention), dX stays fp32

All tensors are [B, H, N, D] (any strides with a unit innermost stride);
the attention output is returned as [B, N, Hq, D] like the reference
(modeling_lucid.py:546).  Head dimensions below 128 (e.g. the 68 of the
reference's lucid/config) are zero-padded to the kernels' 128 columns inside
the autograd functions and sliced back; zero columns change neither the
scores nor the solve, and the kernels take the true D for the RMS mean of
K^.  The stage functions take padded 128-column tensors and the true head
dimension as ``d``.  There is no CPU path: CPU tensors raise.

Run-time failures (a bounded wait inside a kernel that ran out) are read back from
each call's status word without stalling the stream and raised as LucidError at the
next call or by ``check_status()`` (_lib._StatusWatch).
"""
from __future__ import annotations

import os

import torch

from . import _lib

__all__ = [
    "solve_fwd", "attn_fwd", "fused_fwd", "attn_bwd", "solve_bwd",
    "LucidSolveFunction", "LucidAttnFunction", "LucidAttentionFunction",
    "lucid_attention", "padded_len", "decode_update", "decode_attention", "decode_step", "decode_step_fused",
    "stored_tiles_fit", "check_status",
]

check_status = _lib.check_status


def padded_len(n: int) -> int:
    return ((n + 127) // 128) * 128


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _prep(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_cuda:
        raise RuntimeError(f"{name}: LUCID B200 kernels need CUDA tensors (no CPU fallback)")
    if t.dtype != torch.bfloat16:
        raise TypeError(f"{name}: expected bfloat16, got {t.dtype}")
    if t.dim() != 4:
        raise ValueError(f"{name}: expected a 4-D [B, H, N, D] tensor, got shape {tuple(t.shape)}")
    ok = t.stride(-1) == 1 and all(s % 8 == 0 for s in t.stride()[:-1]) and t.data_ptr() % 16 == 0
    return t if ok else t.contiguous()


def _pad128(t: torch.Tensor) -> torch.Tensor:
    d = t.shape[-1]
    if d > 128:
        raise ValueError(f"head dimension {d} > 128 is not supported")
    return t if d == 128 else torch.nn.functional.pad(t, (0, 128 - d))


def _s3(t: torch.Tensor):
    return t.stride(0), t.stride(1), t.stride(2)


def _ws(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def stored_tiles_fit(nbytes: int, device) -> bool:
    """The stored-tile backward schedule (the column pass stores its packed dS^T tiles,
    the row pass streams them instead of recomputing S and dP) trades O(N^2) memory
    for a third of the row pass's tensor work; take it when its workspace fits in
    half of what this process can still allocate.  LUCID_B200_STORED_TILES=0 / 1
    forces the choice."""
    env = os.environ.get("LUCID_B200_STORED_TILES")
    if env is not None:
        return env != "0"
    free, _ = torch.cuda.mem_get_info(device)
    avail = free + torch.cuda.memory_reserved(device) - torch.cuda.memory_allocated(device)
    return nbytes <= 0.5 * avail


# ---------------------------------------------------------------------------
# stages
# ---------------------------------------------------------------------------
def solve_fwd(k: torch.Tensor, v: torch.Tensor, scale: float, eps: float, d: int | None = None):
    """X = P^-1 V.  Returns (x_int, khat, u, rstd, dinv); x_int is
    [B, H, Npad, 128] (rows >= N are padding)."""
    lib = _lib.load()
    _lib.STATUS.poll()
    k = _prep(k, "key")
    v = _prep(v, "value")
    B, H, N, W = k.shape
    D = W if d is None else d
    if v.shape != k.shape:
        raise ValueError(f"key {tuple(k.shape)} and value {tuple(v.shape)} must match")
    Np = padded_len(N)
    dev = k.device
    x = torch.empty(B, H, Np, W, dtype=torch.bfloat16, device=dev)
    khat = torch.empty(B, H, Np, W, dtype=torch.bfloat16, device=dev)
    u = torch.empty(B, H, Np, 128, dtype=torch.bfloat16, device=dev)
    rstd = torch.empty(B, H, Np, dtype=torch.float32, device=dev)
    dinv = torch.empty(B, H, Np, dtype=torch.float32, device=dev)
    # the chain schedule's buffers when the library picks it (few heads), else the flags
    ws = _ws(lib.lucid_solve_fwd_fast_workspace_bytes(B, H, N, D), dev)
    rc = lib.lucid_solve_fwd(B, H, N, D, float(scale), float(eps), k.data_ptr(), *_s3(k),
                             v.data_ptr(), *_s3(v), x.data_ptr(), khat.data_ptr(), u.data_ptr(),
                             rstd.data_ptr(), dinv.data_ptr(), ws.data_ptr(), ws.numel(), _stream())
    _lib.check(rc, "lucid_solve_fwd")
    _lib.STATUS.watch(ws, "lucid_solve_fwd")
    return x, khat, u, rstd, dinv


def fused_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, eps: float, d: int | None = None):
    """solve_fwd then attn_fwd (with the residual) in one library call, which runs them
    as one launch under the solve's chain schedule.  Returns
    (x_int, khat, u, rstd, dinv, o, lse, o_res) as the two stages do."""
    lib = _lib.load()
    _lib.STATUS.poll()
    q = _prep(q, "query")
    k = _prep(k, "key")
    v = _prep(v, "value")
    B, Hq, N, W = q.shape
    Hkv = k.shape[1]
    D = W if d is None else d
    if k.shape != (B, Hkv, N, W) or v.shape != k.shape:
        raise ValueError(f"query {tuple(q.shape)}, key {tuple(k.shape)} and value {tuple(v.shape)} do not match")
    Np = padded_len(N)
    dev = k.device
    x = torch.empty(B, Hkv, Np, W, dtype=torch.bfloat16, device=dev)
    khat = torch.empty(B, Hkv, Np, W, dtype=torch.bfloat16, device=dev)
    u = torch.empty(B, Hkv, Np, 128, dtype=torch.bfloat16, device=dev)
    rstd = torch.empty(B, Hkv, Np, dtype=torch.float32, device=dev)
    dinv = torch.empty(B, Hkv, Np, dtype=torch.float32, device=dev)
    o = torch.empty(B, N, Hq, W, dtype=torch.bfloat16, device=dev)
    ot = o.transpose(1, 2)
    lse = torch.empty(B, Hq, Np, dtype=torch.float32, device=dev)
    o_res = torch.empty_like(o)
    ws = _ws(lib.lucid_fused_fwd_workspace_bytes(B, Hq, Hkv, N, D), dev)
    rc = lib.lucid_fused_fwd(B, Hq, Hkv, N, D, float(scale), float(eps), q.data_ptr(), *_s3(q), k.data_ptr(),
                             *_s3(k), v.data_ptr(), *_s3(v), x.data_ptr(), khat.data_ptr(), u.data_ptr(),
                             rstd.data_ptr(), dinv.data_ptr(), ot.data_ptr(), *_s3(ot), lse.data_ptr(),
                             o_res.data_ptr(), ws.data_ptr(), ws.numel(), _stream())
    _lib.check(rc, "lucid_fused_fwd")
    _lib.STATUS.watch(ws, "lucid_fused_fwd")
    return x, khat, u, rstd, dinv, o, lse, o_res


def attn_fwd(q: torch.Tensor, k: torch.Tensor, x_int: torch.Tensor, scale: float, d: int | None = None,
             residual: bool = False):
    """O = softmax(scale Q K^T + causal) X.  Returns (o [B,N,Hq,128], lse), and with
    ``residual`` also o_res (o's shape): the bf16 rounding residual of the fp32 output,
    which attn_bwd adds back to O for rowsum(dO * O)."""
    lib = _lib.load()
    _lib.STATUS.poll()
    q = _prep(q, "query")
    k = _prep(k, "key")
    B, Hq, N, W = q.shape
    D = W if d is None else d
    Hkv = k.shape[1]
    Np = padded_len(N)
    if k.shape != (B, Hkv, N, W) or x_int.shape != (B, Hkv, Np, W) or not x_int.is_contiguous():
        raise ValueError("attn_fwd: inconsistent shapes")
    dev = q.device
    o = torch.empty(B, N, Hq, W, dtype=torch.bfloat16, device=dev)
    ot = o.transpose(1, 2)
    lse = torch.empty(B, Hq, Np, dtype=torch.float32, device=dev)
    o_res = torch.empty_like(o) if residual else None
    ws = _ws(lib.lucid_attn_fwd_workspace_bytes(B, Hq, Hkv, N, D), dev)
    rc = lib.lucid_attn_fwd(B, Hq, Hkv, N, D, float(scale), q.data_ptr(), *_s3(q), k.data_ptr(),
                            *_s3(k), x_int.data_ptr(), ot.data_ptr(), *_s3(ot), lse.data_ptr(),
                            o_res.data_ptr() if residual else None, ws.data_ptr(), ws.numel(), _stream())
    _lib.check(rc, "lucid_attn_fwd")
    _lib.STATUS.watch(ws, "lucid_attn_fwd")
    return (o, lse, o_res) if residual else (o, lse)


def attn_bwd(q, k, x_int, o, do, lse, scale: float, d: int | None = None, o_res=None):
    """Backward of attn_fwd.  o, do (and o_res, attn_fwd's residual, if given) are
    [B,N,Hq,128].  Returns (dq [B,Hq,N,128] bf16, dk_f32 [B,Hkv,Npad,128],
    dx_f32 [B,Hkv,Npad,128])."""
    lib = _lib.load()
    _lib.STATUS.poll()
    q = _prep(q, "query")
    k = _prep(k, "key")
    ot = _prep(o.transpose(1, 2), "attn_output")
    dot = _prep(do.transpose(1, 2), "grad_output")
    if o_res is not None and o_res.stride() != o.stride():
        raise ValueError("attn_bwd: o_res must have o's layout")
    B, Hq, N, W = q.shape
    D = W if d is None else d
    Hkv = k.shape[1]
    Np = padded_len(N)
    dev = q.device
    dq = torch.empty(B, Hq, N, W, dtype=torch.bfloat16, device=dev)
    dk = torch.empty(B, Hkv, Np, W, dtype=torch.float32, device=dev)
    dx = torch.empty(B, Hkv, Np, W, dtype=torch.float32, device=dev)
    nbytes = lib.lucid_attn_bwd_workspace_bytes(B, Hq, Hkv, N, D)
    fast = lib.lucid_attn_bwd_fast_workspace_bytes(B, Hq, Hkv, N, D)
    ws = _ws(fast if stored_tiles_fit(fast, dev) else nbytes, dev)
    rc = lib.lucid_attn_bwd(B, Hq, Hkv, N, D, float(scale), q.data_ptr(), *_s3(q), k.data_ptr(),
                            *_s3(k), x_int.data_ptr(), ot.data_ptr(), *_s3(ot), dot.data_ptr(),
                            *_s3(dot), lse.data_ptr(), o_res.data_ptr() if o_res is not None else None,
                            dq.data_ptr(), *_s3(dq), dk.data_ptr(),
                            dx.data_ptr(), ws.data_ptr(), ws.numel(), _stream())
    _lib.check(rc, "lucid_attn_bwd")
    _lib.STATUS.watch(ws, "lucid_attn_bwd")
    return dq, dk, dx


def solve_bwd(k, x_int, khat, u, rstd, dinv, dx_f32, scale: float, dk_add=None, d: int | None = None):
    """Backward of solve_fwd.  Returns (dk, dv) bf16 [B,H,N,128]."""
    lib = _lib.load()
    _lib.STATUS.poll()
    k = _prep(k, "key")
    B, H, N, W = k.shape
    D = W if d is None else d
    dev = k.device
    dk = torch.empty(B, H, N, W, dtype=torch.bfloat16, device=dev)
    dv = torch.empty(B, H, N, W, dtype=torch.bfloat16, device=dev)
    nbytes = lib.lucid_solve_bwd_workspace_bytes(B, H, N, D)
    fast = lib.lucid_solve_bwd_fast_workspace_bytes(B, H, N, D)
    ws = _ws(fast if stored_tiles_fit(fast, dev) else nbytes, dev)
    rc = lib.lucid_solve_bwd(B, H, N, D, float(scale), k.data_ptr(), *_s3(k), x_int.data_ptr(),
                             khat.data_ptr(), u.data_ptr(), rstd.data_ptr(), dinv.data_ptr(),
                             dx_f32.data_ptr(), dk_add.data_ptr() if dk_add is not None else None,
                             dk.data_ptr(), *_s3(dk), dv.data_ptr(), *_s3(dv), ws.data_ptr(), ws.numel(),
                             _stream())
    _lib.check(rc, "lucid_solve_bwd")
    _lib.STATUS.watch(ws, "lucid_solve_bwd")
    return dk, dv


# ---------------------------------------------------------------------------
# autograd
# ---------------------------------------------------------------------------
class LucidSolveFunction(torch.autograd.Function):
    """X = P^-1 V (get_v_prime, exp_k_norm branch).  Returns X [B,H,N,D]."""

    @staticmethod
    def forward(ctx, key, value, scaling: float, eps: float):
        D = key.shape[-1]
        k = _prep(_pad128(key), "key")
        x, khat, u, rstd, dinv = solve_fwd(k, _pad128(value), scaling, eps, d=D)
        ctx.save_for_backward(k, x, khat, u, rstd, dinv)
        ctx.scaling, ctx.d = scaling, D
        return x[:, :, : k.shape[2], :D]

    @staticmethod
    def backward(ctx, gx):
        k, x, khat, u, rstd, dinv = ctx.saved_tensors
        B, H, N, W = k.shape
        D = ctx.d
        dx = torch.zeros(B, H, x.shape[2], W, dtype=torch.float32, device=k.device)
        dx[:, :, :N, :D] = gx.float()
        dk, dv = solve_bwd(k, x, khat, u, rstd, dinv, dx, ctx.scaling, d=D)
        return dk[..., :D], dv[..., :D], None, None


class LucidAttnFunction(torch.autograd.Function):
    """O = softmax(s Q K^T + causal) X (eager_lucid_attention_forward).
    Returns O as [B, N, Hq, D]."""

    @staticmethod
    def forward(ctx, query, key, v_prime, scaling: float):
        B, Hkv, N, D = key.shape
        q, k = _pad128(query), _pad128(key)
        x = torch.zeros(B, Hkv, padded_len(N), 128, dtype=torch.bfloat16, device=key.device)
        x[:, :, :N, :D] = v_prime
        o, lse, o_res = attn_fwd(q, k, x, scaling, d=D, residual=True)
        ctx.save_for_backward(q, k, x, o, lse, o_res)
        ctx.scaling, ctx.d = scaling, D
        return o[..., :D]

    @staticmethod
    def backward(ctx, do):
        q, k, x, o, lse, o_res = ctx.saved_tensors
        N, D = k.shape[2], ctx.d
        dq, dk, dx = attn_bwd(q, k, x, o, _pad128(do), lse, ctx.scaling, d=D, o_res=o_res)
        return (dq[..., :D], dk[:, :, :N, :D].to(torch.bfloat16), dx[:, :, :N, :D].to(torch.bfloat16), None)


class LucidAttentionFunction(torch.autograd.Function):
    """Fused LUCID attention: O = softmax(s Q K^T + causal) P^-1 V, returned
    as [B, N, Hq, D]; q [B,Hq,N,D], k, v [B,Hkv,N,D]."""

    @staticmethod
    def forward(ctx, query, key, value, scaling: float, eps: float):
        D = key.shape[-1]
        k = _prep(_pad128(key), "key")
        q = _prep(_pad128(query), "query")
        x, khat, u, rstd, dinv, o, lse, o_res = fused_fwd(q, k, _pad128(value), scaling, eps, d=D)
        ctx.save_for_backward(q, k, x, khat, u, rstd, dinv, o, lse, o_res)
        ctx.scaling, ctx.d = scaling, D
        return o if D == 128 else o[..., :D]

    @staticmethod
    def backward(ctx, do):
        q, k, x, khat, u, rstd, dinv, o, lse, o_res = ctx.saved_tensors
        s, D = ctx.scaling, ctx.d
        dq, dk_attn, dx = attn_bwd(q, k, x, o, _pad128(do), lse, s, d=D, o_res=o_res)
        dk, dv = solve_bwd(k, x, khat, u, rstd, dinv, dx, s, dk_add=dk_attn, d=D)
        if D == 128:
            return dq, dk, dv, None, None
        return dq[..., :D], dk[..., :D], dv[..., :D], None, None


def lucid_attention(query, key, value, scaling: float | None = None, eps: float = 1e-5):
    """Fused LUCID attention.  query [B,Hq,N,D], key/value [B,Hkv,N,D]
    (bf16, CUDA).  Returns O [B, N, Hq, D]."""
    if scaling is None:
        scaling = query.shape[-1] ** -0.5
    return LucidAttentionFunction.apply(query, key, value, float(scaling), float(eps))


# ---------------------------------------------------------------------------
# decode (inference with a key / solved-value cache)
# ---------------------------------------------------------------------------
def _prep_dec(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_cuda:
        raise RuntimeError(f"{name}: LUCID B200 kernels need CUDA tensors (no CPU fallback)")
    if t.dtype != torch.bfloat16:
        raise TypeError(f"{name}: expected bfloat16, got {t.dtype}")
    ok = t.stride(-1) == 1 and all(s % 4 == 0 for s in t.stride()[:-1]) and t.data_ptr() % 8 == 0
    return t if ok else t.contiguous()


def decode_update(key: torch.Tensor, value: torch.Tensor, key_cache: torch.Tensor, x_cache: torch.Tensor,
                  scale: float, eps: float = 1e-5) -> torch.Tensor:
    """get_new_v_prime (modeling_lucid.py:576-598): x_new = value -
    exp(s k^ K^_cache^T - 1/s) X_cache, key/value [B,H,Ln,D], caches
    [B,H,Nc,D] (raw keys, solved values; D <= 128 a multiple of 4, no
    padding).  Returns x_new [B,H,Ln,D]."""
    lib = _lib.load()
    key, value = _prep_dec(key, "key"), _prep_dec(value, "value")
    key_cache, x_cache = _prep_dec(key_cache, "key_cache"), _prep_dec(x_cache, "value_cache")
    B, H, Ln, D = key.shape
    Nc = key_cache.shape[2]
    out = torch.empty(B, H, Ln, D, dtype=torch.bfloat16, device=key.device)
    ws = _ws(lib.lucid_decode_workspace_bytes(B, H, Ln, Nc, D), key.device)
    rc = lib.lucid_decode_update(B, H, Ln, Nc, D, float(scale), float(eps), key.data_ptr(), *_s3(key),
                                 value.data_ptr(), *_s3(value), key_cache.data_ptr(), *_s3(key_cache),
                                 x_cache.data_ptr(), *_s3(x_cache), out.data_ptr(), *_s3(out),
                                 ws.data_ptr(), ws.numel(), _stream())
    _lib.check(rc, "lucid_decode_update")
    return out


def decode_attention(query: torch.Tensor, key_cache: torch.Tensor, x_cache: torch.Tensor,
                     scale: float) -> torch.Tensor:
    """softmax(s Q K^T + causal) X for Ln new queries at the end of the cache
    (eager_lucid_attention_forward during decoding).  query [B,Hq,Ln,D],
    caches [B,Hkv,Nc,D] already holding the new tokens (D <= 128 a multiple
    of 4).  Returns O as [B, Ln, Hq, D] like the reference (modeling_lucid.py:546)."""
    lib = _lib.load()
    query = _prep_dec(query, "query")
    key_cache, x_cache = _prep_dec(key_cache, "key_cache"), _prep_dec(x_cache, "value_cache")
    B, Hq, Ln, D = query.shape
    Hkv, Nc = key_cache.shape[1], key_cache.shape[2]
    o = torch.empty(B, Ln, Hq, D, dtype=torch.bfloat16, device=query.device)
    ov = o.transpose(1, 2)
    ws = _ws(lib.lucid_decode_attn_workspace_bytes(B, Hq, Ln, Nc, D), query.device)
    rc = lib.lucid_decode_attn(B, Hq, Hkv, Ln, Nc, D, float(scale), query.data_ptr(), *_s3(query),
                               key_cache.data_ptr(), *_s3(key_cache), x_cache.data_ptr(), *_s3(x_cache),
                               ov.data_ptr(), *_s3(ov), ws.data_ptr(), ws.numel(), _stream())
    _lib.check(rc, "lucid_decode_attn")
    return o


def decode_step_fused(num_heads: int, num_kv_heads: int, new_tokens: int) -> bool:
    """True when decode_step has a single-pass kernel for this shape (one new token
    with 1 or 2 query heads per kv head, or two new tokens without grouping)."""
    return bool(_lib.load().lucid_decode_step_fused(num_heads, num_kv_heads, new_tokens))


def decode_step(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, key_cache: torch.Tensor,
                x_cache: torch.Tensor, scale: float, eps: float = 1e-5):
    """One decoding step of LucidAttention.forward (modeling_lucid.py:467-481, then
    :505-549) in one pass over the cache: x_new = get_new_v_prime(key, value) against
    the cache and the attention of the new queries over [cache; new tokens].
    query [B,Hq,Ln,D], key / value [B,Hkv,Ln,D], caches [B,Hkv,Nc,D] holding the
    tokens before this step (raw keys, solved values).  Returns (O [B,Ln,Hq,D],
    x_new [B,Hkv,Ln,D]); the caller appends (key, x_new) to its cache.  Shapes
    without a fused kernel (decode_step_fused false) raise."""
    lib = _lib.load()
    query, key, value = _prep_dec(query, "query"), _prep_dec(key, "key"), _prep_dec(value, "value")
    key_cache, x_cache = _prep_dec(key_cache, "key_cache"), _prep_dec(x_cache, "value_cache")
    B, Hq, Ln, D = query.shape
    Hkv, Nc = key_cache.shape[1], key_cache.shape[2]
    x_new = torch.empty(B, Hkv, Ln, D, dtype=torch.bfloat16, device=query.device)
    o = torch.empty(B, Ln, Hq, D, dtype=torch.bfloat16, device=query.device)
    ov = o.transpose(1, 2)
    ws = _ws(lib.lucid_decode_step_workspace_bytes(B, Hq, Hkv, Ln, Nc, D), query.device)
    rc = lib.lucid_decode_step(B, Hq, Hkv, Ln, Nc, D, float(scale), float(eps), query.data_ptr(), *_s3(query),
                               key.data_ptr(), *_s3(key), value.data_ptr(), *_s3(value),
                               key_cache.data_ptr(), *_s3(key_cache), x_cache.data_ptr(), *_s3(x_cache),
                               x_new.data_ptr(), *_s3(x_new), ov.data_ptr(), *_s3(ov),
                               ws.data_ptr(), ws.numel(), _stream())
    _lib.check(rc, "lucid_decode_step")
    return o, x_new
