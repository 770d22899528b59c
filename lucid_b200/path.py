"""LUCID-Path on the B200 kernels: the drop-in for
``parallel_lucid_path_attention`` (lucid_path/triton_code/parallel.py:180-241).

    o, k_cache = parallel_lucid_path_attention(k, v, w, beta, q=None, g=None,
                                               scale=None, cu_seqlens=None,
                                               use_cache=False)

solves (I + L) O = V with L = stril(exp(scale * A - 1/scale)) and the
Householder-path scores A_rc = q_r^T (H_r ... H_{c+1}) k_c,
H_t = I - beta_t w_t w_t^T.  Layout is the reference's BTHD: k, v, w
[B, T, H, K], beta [B, T, H], q [B, T, HQ, K] (defaults to k), o [B, T, HQ, V].

The forward and backward are the C-ABI entry points lucid_path_fwd /
lucid_path_bwd (include/lucid_b200.h); the forward's workspace is the state
saved for the backward.  There is no CPU path: CPU tensors raise.

Head dimensions: 16, 32, 64 or 128 as in the reference (parallel.py:230-231).
The kernels are 128 wide; a smaller head dimension is zero-padded to 128 and
the outputs sliced back, which is exact: with zero columns in w every
Householder H_t acts as the identity on them, so q, k and v stay zero there
and the scores are unchanged.  ``g`` must be None (the reference asserts the
same, :235).  ``cu_seqlens`` (packed variable-length batches, B == 1) runs the
sequences with the same number of 128-token blocks as one batch, each zero-padded
at its end (exact for the real tokens; see _varlen).
"""
from __future__ import annotations

import os

import torch

from . import _lib

__all__ = ["parallel_lucid_path_attention", "ParallelLUCIDPathAttentionFunction", "path_fwd", "path_bwd",
           "parallel_path_attention_fwd", "path_memory_groups", "PathArgumentError"]


class PathArgumentError(ValueError, AssertionError):
    """An argument the reference op rejects.  The reference checks its arguments with
    ``assert`` (parallel.py:230-239), so this is an AssertionError for callers written
    against it, and a ValueError for everyone else."""


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _prep(t: torch.Tensor, name: str, ndim: int = 4) -> torch.Tensor:
    if not t.is_cuda:
        raise RuntimeError(f"{name}: LUCID B200 kernels need CUDA tensors (no CPU fallback)")
    if t.dim() != ndim:
        raise ValueError(f"{name}: expected a {ndim}-D tensor, got shape {tuple(t.shape)}")
    if ndim == 4:
        if t.dtype != torch.bfloat16:
            raise TypeError(f"{name}: expected bfloat16, got {t.dtype}")
        ok = t.stride(-1) == 1 and all(s % 8 == 0 for s in t.stride()[:-1]) and t.data_ptr() % 16 == 0
        return t if ok else t.contiguous()
    if t.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError(f"{name}: expected bfloat16 or float32, got {t.dtype}")
    return t


def _s3(t: torch.Tensor):
    return t.stride(0), t.stride(1), t.stride(2)


def _ws(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def path_fwd(k, v, w, beta, q=None, scale=None, use_cache=False):
    """Forward stage.  Returns (o [B,T,HQ,V], state, k_cache); ``state`` is the
    forward workspace the backward reads; ``k_cache`` ([B,T,H,K], the keys
    transformed by every later Householder, prepare_k_cache.py) or None."""
    lib = _lib.load()
    _lib.STATUS.poll()
    k, v, w = _prep(k, "k"), _prep(v, "v"), _prep(w, "w")
    beta = _prep(beta, "beta", 3)
    B, T, H, K = k.shape
    if K != 128 or v.shape[-1] != 128:
        raise NotImplementedError("LUCID-Path B200 kernels support head_dim 128 only")
    if w.shape != k.shape or v.shape[:3] != k.shape[:3] or tuple(beta.shape) != (B, T, H):
        raise ValueError("k, v, w must be [B, T, H, 128] and beta [B, T, H]")
    if q is not None:
        q = _prep(q, "q")
        if q.shape[0] != B or q.shape[1] != T or q.shape[3] != K or q.shape[2] % H != 0:
            raise ValueError("q must be [B, T, HQ, 128] with HQ a multiple of H")
    HQ = q.shape[2] if q is not None else H
    s = float(K ** -0.5 if scale is None else scale)
    dev = k.device
    o = torch.empty(B, T, HQ, v.shape[-1], dtype=v.dtype, device=dev)
    kc = torch.empty(B, T, H, K, dtype=k.dtype, device=dev) if use_cache else None
    kcp, kcs = (kc.data_ptr(), _s3(kc)) if kc is not None else (None, (0, 0, 0))
    ws = _ws(lib.lucid_path_fwd_workspace_bytes(B, T, H, HQ, K), dev)
    qp, qs = (q.data_ptr(), _s3(q)) if q is not None else (None, (0, 0, 0))
    rc = lib.lucid_path_fwd(B, T, H, HQ, K, s, qp, *qs, k.data_ptr(), *_s3(k), v.data_ptr(), *_s3(v),
                            w.data_ptr(), *_s3(w), beta.data_ptr(), int(beta.dtype == torch.float32), *beta.stride(),
                            o.data_ptr(), *_s3(o), kcp, *kcs, ws.data_ptr(), ws.numel(), _stream())
    _lib.check(rc, "lucid_path_fwd")
    _lib.STATUS.watch(ws, "lucid_path_fwd")
    return o, ws, kc


def path_bwd(state, do, k, w, beta, q=None, scale=None):
    """Backward stage.  Returns (dq or None, dk, dv, dw, dbeta); with q None
    the query gradient is folded into dk (q = k)."""
    lib = _lib.load()
    _lib.STATUS.poll()
    k, w, do = _prep(k, "k"), _prep(w, "w"), _prep(do, "do")
    beta = _prep(beta, "beta", 3)
    B, T, H, K = k.shape
    HQ = q.shape[2] if q is not None else H
    s = float(K ** -0.5 if scale is None else scale)
    dev = k.device
    dk = torch.empty(B, T, H, K, dtype=k.dtype, device=dev)
    dv = torch.empty(B, T, H, K, dtype=k.dtype, device=dev)
    dw = torch.empty(B, T, H, K, dtype=w.dtype, device=dev)
    dbeta = torch.empty(B, T, H, dtype=beta.dtype, device=dev)
    dq = None
    if q is not None:
        q = _prep(q, "q")
        dq = torch.empty(B, T, HQ, K, dtype=q.dtype, device=dev)
    ws = _ws(lib.lucid_path_bwd_workspace_bytes(B, T, H, HQ, K), dev)
    qp, qs = (q.data_ptr(), _s3(q)) if q is not None else (None, (0, 0, 0))
    dqp, dqs = (dq.data_ptr(), _s3(dq)) if dq is not None else (None, (0, 0, 0))
    rc = lib.lucid_path_bwd(B, T, H, HQ, K, s, qp, *qs, k.data_ptr(), *_s3(k), w.data_ptr(), *_s3(w),
                            beta.data_ptr(), int(beta.dtype == torch.float32), *beta.stride(),
                            do.data_ptr(), *_s3(do), state.data_ptr(), state.numel(),
                            dqp, *dqs, dk.data_ptr(), *_s3(dk), dv.data_ptr(), *_s3(dv), dw.data_ptr(), *_s3(dw),
                            dbeta.data_ptr(), int(dbeta.dtype == torch.float32), *dbeta.stride(),
                            ws.data_ptr(), ws.numel(), _stream())
    _lib.check(rc, "lucid_path_bwd")
    _lib.STATUS.watch(ws, "lucid_path_bwd")
    return dq, dk, dv, dw, dbeta


def path_memory_groups(B: int, T: int, H: int, HQ: int, device, budget: int | None = None):
    """The (batch, kv-head) slices the op runs at once.  The forward's saved state and the
    backward's workspace hold O(T^2) block-pair tiles per (batch, query head) (about
    4 x 32 KB per pair of 128-row blocks); when the whole batch's tiles do not fit in
    ``budget`` bytes (default: half of what this process can still allocate;
    LUCID_B200_PATH_MAX_BYTES overrides), the op runs kv-head groups one after another
    and the backward recomputes each group's forward, so memory is bounded by one
    group.  Returns a list of (b0, b1, h0, h1) kv-head slices; raises if a single kv
    head does not fit."""
    lib = _lib.load()
    per = lambda b, h: (lib.lucid_path_fwd_workspace_bytes(b, T, h, h * (HQ // H), 128) +
                        lib.lucid_path_bwd_workspace_bytes(b, T, h, h * (HQ // H), 128))
    if budget is None:
        env = os.environ.get("LUCID_B200_PATH_MAX_BYTES")
        if env is not None:
            budget = int(env)
        else:
            free, _ = torch.cuda.mem_get_info(device)
            budget = int(0.5 * (free + torch.cuda.memory_reserved(device) - torch.cuda.memory_allocated(device)))
    if per(B, H) <= budget:
        return [(0, B, 0, H)]
    if per(1, 1) > budget:
        raise _lib.LucidError(f"LUCID-Path at T={T}: one head needs {per(1, 1) / 2**30:.1f} GiB of block-pair "
                              f"workspace, more than the {budget / 2**30:.1f} GiB available")
    hg = max(h for h in range(1, H + 1) if H % h == 0 and per(1, h) <= budget)
    return [(b, b + 1, h0, h0 + hg) for b in range(B) for h0 in range(0, H, hg)]


class ParallelLUCIDPathAttentionFunction(torch.autograd.Function):
    """Autograd mirror of parallel.py:27-177 (same positional arguments).  When the
    block-pair workspace of the whole batch does not fit (path_memory_groups), kv-head
    groups run one after another and the backward recomputes each group's forward."""

    @staticmethod
    def forward(ctx, q, k, v, w, beta, g, scale, cu_seqlens, use_cache=False):
        if g is not None:
            raise NotImplementedError("g is not supported (the reference asserts g is None)")
        q_given = q is not None and q is not k
        _prep(k, "k")   # CPU tensors raise here, before any device query
        B, T, H, _ = k.shape
        HQ = q.shape[2] if q_given else H
        groups = path_memory_groups(B, T, H, HQ, k.device)
        ctx.q_given = q_given
        ctx.q_is_k = q is k
        ctx.scale = scale
        ctx.groups = groups
        if len(groups) == 1:
            o, state, kc = path_fwd(k, v, w, beta, q=q if q_given else None, scale=scale, use_cache=use_cache)
            ctx.save_for_backward(q if q_given else None, k, v, w, beta, state)
        else:
            G = HQ // H
            o = torch.empty(B, T, HQ, v.shape[-1], dtype=v.dtype, device=k.device)
            kc = torch.empty_like(k) if use_cache else None
            for b0, b1, h0, h1 in groups:
                sl, slq = (slice(b0, b1), slice(None), slice(h0, h1)), (slice(b0, b1), slice(None), slice(h0 * G, h1 * G))
                og, _, kcg = path_fwd(k[sl], v[sl], w[sl], beta[sl], q=q[slq] if q_given else None, scale=scale,
                                      use_cache=use_cache)
                o[slq] = og
                if use_cache:
                    kc[sl] = kcg
                del og, kcg
            ctx.save_for_backward(q if q_given else None, k, v, w, beta, None)
        if kc is not None:
            ctx.mark_non_differentiable(kc)
        return o, kc

    @staticmethod
    def backward(ctx, do, dk_cache):
        q, k, v, w, beta, state = ctx.saved_tensors
        if len(ctx.groups) == 1:
            dq, dk, dv, dw, dbeta = path_bwd(state, do, k, w, beta, q=q, scale=ctx.scale)
        else:
            H, HQ = k.shape[2], (q.shape[2] if q is not None else k.shape[2])
            G = HQ // H
            dq = torch.empty_like(q) if q is not None else None
            dk, dv, dw = torch.empty_like(k), torch.empty_like(v), torch.empty_like(w)
            dbeta = torch.empty_like(beta)
            for b0, b1, h0, h1 in ctx.groups:
                sl, slq = (slice(b0, b1), slice(None), slice(h0, h1)), (slice(b0, b1), slice(None), slice(h0 * G, h1 * G))
                qg = q[slq] if q is not None else None
                _, st, _ = path_fwd(k[sl], v[sl], w[sl], beta[sl], q=qg, scale=ctx.scale)   # recompute the state
                r = path_bwd(st, do[slq], k[sl], w[sl], beta[sl], q=qg, scale=ctx.scale)
                del st
                if dq is not None:
                    dq[slq] = r[0]
                dk[sl], dv[sl], dw[sl], dbeta[sl] = r[1], r[2], r[3], r[4]
        if ctx.q_is_k:
            # q and k are the same tensor: the reference returns dq and dk
            # separately and autograd sums them; dk already holds the sum.
            return None, dk, dv, dw, dbeta, None, None, None, None
        return dq, dk, dv, dw, dbeta, None, None, None, None


_HEAD_DIMS = (16, 32, 64, 128)


def _pad128(t):
    return t if t.shape[-1] == 128 else torch.nn.functional.pad(t, (0, 128 - t.shape[-1]))


def parallel_lucid_path_attention(k, v, w, beta, q=None, g=None, scale=None, cu_seqlens=None, use_cache=False):
    """Drop-in for lucid_path/triton_code/parallel.py:180-241; returns (o, k_cache).
    k_cache is None unless use_cache (then the keys transformed by every later
    Householder, prepare_k_cache.py:8-74; no gradient flows through it, as in
    the reference, whose backward ignores dk_new)."""
    if q is None:
        q = k
    if scale is None:
        scale = k.shape[-1] ** -0.5
    if q.shape[-1] not in _HEAD_DIMS or v.shape[-1] not in _HEAD_DIMS:
        raise PathArgumentError("only support head_dim in [16, 32, 64, 128]")
    if q.shape[-1] != k.shape[-1]:
        raise PathArgumentError("q, k should have the same head_dim.")
    if k.shape != w.shape:
        raise PathArgumentError("k, w should have the same shape.")
    if beta.shape[:3] != k.shape[:3]:
        raise PathArgumentError("beta should have the same number of heads as k")
    if g is not None:
        raise PathArgumentError("g is not supported")
    if q.shape[-2] % k.shape[-2] != 0:
        raise PathArgumentError("the number of query heads should be divisible by the number of key heads")
    K, V = k.shape[-1], v.shape[-1]
    if K < 128 or V < 128:
        o, kc = parallel_lucid_path_attention(_pad128(k), _pad128(v), _pad128(w), beta,
                                              q=None if q is k else _pad128(q), scale=scale,
                                              cu_seqlens=cu_seqlens, use_cache=use_cache)
        return o[..., :V], (kc[..., :K] if kc is not None else None)
    if cu_seqlens is None:
        return ParallelLUCIDPathAttentionFunction.apply(q, k, v, w, beta, None, float(scale), None, bool(use_cache))
    if k.shape[0] != 1:
        raise PathArgumentError("cu_seqlens requires a packed batch of size 1")
    return _varlen(q, k, v, w, beta, float(scale), [int(x) for x in cu_seqlens.tolist()], bool(use_cache))


def _varlen(q, k, v, w, beta, scale, bounds, use_cache):
    """Packed variable-length sequences (cu_seqlens = bounds): the sequences with the
    same number of 128-token blocks run as one batch, each zero-padded at its end to
    that block count (one kernel chain per distinct block count instead of one per
    sequence).  Zero padding is exact for the real tokens: a padded token has w = 0 and
    beta = 0 (its Householder is the identity) and comes after every real token of its
    sequence, so causality keeps it out of their outputs, and with dO = 0 there its dV,
    and so its share of every gradient, is zero."""
    T = k.shape[1]
    dev = k.device
    lens = [b - a for a, b in zip(bounds[:-1], bounds[1:])]
    if bounds[0] != 0 or bounds[-1] != T or any(n < 0 for n in lens):
        raise PathArgumentError("cu_seqlens must rise from 0 to the packed length")
    groups = {}
    for s_, n in enumerate(lens):
        if n > 0:
            groups.setdefault((n + 127) // 128, []).append(s_)
    zero_row = lambda t: torch.cat([t[0], t.new_zeros((1,) + tuple(t.shape[2:]))], 0)   # [T + 1, ...]
    qz = zero_row(q) if q is not k else None
    kz, vz, wz, bz = zero_row(k), zero_row(v), zero_row(w), zero_row(beta)
    o_parts, kc_parts, pos = [], [], torch.empty(T, dtype=torch.long)
    base = 0
    for nb, seqs in sorted(groups.items()):
        Tp = nb * 128
        idx = torch.full((len(seqs), Tp), T, dtype=torch.long)   # T: the appended zero row
        for r_, s_ in enumerate(seqs):
            a, n = bounds[s_], lens[s_]
            idx[r_, :n] = torch.arange(a, a + n)
            pos[a:a + n] = base + r_ * Tp + torch.arange(n)
        base += len(seqs) * Tp
        idx = idx.to(dev)
        kk = kz[idx]
        o, kc = ParallelLUCIDPathAttentionFunction.apply(qz[idx] if qz is not None else kk, kk, vz[idx], wz[idx],
                                                         bz[idx], None, scale, None, use_cache)
        o_parts.append(o.reshape((-1,) + tuple(o.shape[2:])))
        if use_cache:
            kc_parts.append(kc.reshape((-1,) + tuple(kc.shape[2:])))
    pos = pos.to(dev)
    o = torch.cat(o_parts, 0)[pos].unsqueeze(0)
    kc = torch.cat(kc_parts, 0)[pos].unsqueeze(0) if use_cache else None
    return o, kc


def parallel_path_attention_fwd(q, k, v, w, beta, scale=None):
    """PaTH softmax attention forward: o [B,T,HQ,V] and the log2-sum-exp lse
    [B,T,HQ] (float32), the outputs of the reference's
    intra_chunk_preprocess_fwd_fn + parallel_path_fwd_fn
    (intra_chunk_preprocess_fwd.py:124-168, parallel_path_fwd.py:127-170).
    ``q`` may be None (q = k).  Forward only: the reference has no backward
    kernels for this op.  Head dimensions below 128 run zero-padded."""
    Kd, Vd = k.shape[-1], v.shape[-1]
    if Kd not in _HEAD_DIMS or Vd not in _HEAD_DIMS:
        raise PathArgumentError("only support head_dim in [16, 32, 64, 128]")
    if Kd < 128 or Vd < 128:
        o, lse = parallel_path_attention_fwd(None if q is None else _pad128(q), _pad128(k), _pad128(v),
                                             _pad128(w), beta, scale=Kd ** -0.5 if scale is None else scale)
        return o[..., :Vd], lse
    lib = _lib.load()
    _lib.STATUS.poll()
    k, v, w = _prep(k, "k"), _prep(v, "v"), _prep(w, "w")
    beta = _prep(beta, "beta", 3)
    B, T, H, K = k.shape
    if K != 128 or v.shape[-1] != 128:
        raise NotImplementedError("PaTH attention B200 kernels support head_dim 128 only")
    if w.shape != k.shape or v.shape[:3] != k.shape[:3] or tuple(beta.shape) != (B, T, H):
        raise ValueError("k, v, w must be [B, T, H, 128] and beta [B, T, H]")
    if q is not None:
        q = _prep(q, "q")
        if q.shape[0] != B or q.shape[1] != T or q.shape[3] != K or q.shape[2] % H != 0:
            raise ValueError("q must be [B, T, HQ, 128] with HQ a multiple of H")
    HQ = q.shape[2] if q is not None else H
    s = float(K ** -0.5 if scale is None else scale)
    dev = k.device
    o = torch.empty(B, T, HQ, v.shape[-1], dtype=v.dtype, device=dev)
    lse = torch.empty(B, T, HQ, dtype=torch.float32, device=dev)
    ws = _ws(lib.lucid_path_attn_fwd_workspace_bytes(B, T, H, HQ, K), dev)
    qp, qs = (q.data_ptr(), _s3(q)) if q is not None else (None, (0, 0, 0))
    rc = lib.lucid_path_attn_fwd(B, T, H, HQ, K, s, qp, *qs, k.data_ptr(), *_s3(k), v.data_ptr(), *_s3(v),
                                 w.data_ptr(), *_s3(w), beta.data_ptr(), int(beta.dtype == torch.float32),
                                 *beta.stride(), o.data_ptr(), *_s3(o), lse.data_ptr(), *lse.stride(),
                                 ws.data_ptr(), ws.numel(), _stream())
    _lib.check(rc, "lucid_path_attn_fwd")
    _lib.STATUS.watch(ws, "lucid_path_attn_fwd")
    return o, lse
