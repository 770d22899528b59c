"""Float32 LUCID reference at full sequence lengths — TEST INFRASTRUCTURE ONLY.

Only tests/ and bench.py's reference measurements may import this module, as
the checker; the product path (lucid_b200) never calls it.

The reference's own training path for one LUCID layer (saisuryadv/LUCID,
modeling_lucid.py) in float32 torch, on whatever device its tensors live
(tests run it on the GPU, so that 32K-128K sequences finish in seconds):

  solve, dense branch N < 2**16     get_v_prime (:551-574): P = tril(exp(s K^K^T - 1/s)),
                                    torch.linalg.solve_triangular(P, V, upper=False)
  solve, blockwise N >= 2**16       Lucid_Tril_Solver.forward (:285-312), row blocks of
                                    BS = 2**14: R_i = V_i - sum_{j<i} exp(s K^_i K^_j^T - 1/s) X_j,
                                    X_i = solve_triangular(tril(exp(s K^_i K^_i^T - 1/s)), R_i)
  attention                         eager_lucid_attention_forward (:505-549): causal softmax
                                    attention in float32 (no TF32), here in query chunks so the
                                    N x N scores never exist at once
  backward                          the analytic gradients torch autograd derives for the dense
                                    branch, in the block form of Lucid_Tril_Solver.backward
                                    (:314-382): dV = P^-T dX by block back substitution,
                                    dK^ = -s [(dV X^T o P) K^ + (X dV^T o P^T) K^], then the
                                    RMSNorm backward (:409, no affine) and the attention's dK.

Tensors are one batch element: q [Hq, N, D], k, v [Hkv, N, D], do [Hq, N, D]
(float32).  With the block size set to N the solve is exactly the dense branch.
tests/test_oracle.py checks this module against the float64 numpy oracle
(oracle/lucid_oracle.py), which the reference's own fixtures pin.
"""
from __future__ import annotations

import torch

__all__ = ["BS_REFERENCE", "reference_block_size", "rms_norm", "solve_fwd", "attention_fwd", "attention_bwd",
           "solve_bwd", "lucid_fwd_bwd"]

# Lucid_Tril_Solver's block size and the length from which get_v_prime takes it
# (modeling_lucid.py:561-572).
BS_REFERENCE = 2 ** 14
BLOCKWISE_FROM = 2 ** 16


def reference_block_size(n: int) -> int:
    """Row-block size of the reference's solve at sequence length n: the dense
    branch (one block) below 2**16, Lucid_Tril_Solver's 2**14 from there on."""
    return n if n < BLOCKWISE_FROM else BS_REFERENCE


def _no_tf32():
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False


def rms_norm(k: torch.Tensor, eps: float):
    """K^ and r = (mean K^2 + eps)^-1/2 (nn.RMSNorm without affine, modeling_lucid.py:409)."""
    r = torch.rsqrt(k.pow(2).mean(-1, keepdim=True) + eps)
    return k * r, r


def _exp_block(a: torch.Tensor, b: torch.Tensor, s: float, diag: bool) -> torch.Tensor:
    e = torch.matmul(a, b.transpose(-1, -2)).mul_(s).sub_(1.0 / s).exp_()
    return torch.tril(e) if diag else e


def solve_fwd(kh: torch.Tensor, v: torch.Tensor, s: float, bs: int) -> torch.Tensor:
    """X = P^-1 V by row blocks of bs (bs >= N: the dense branch)."""
    _no_tf32()
    n = kh.shape[-2]
    x = torch.empty_like(v)
    for i0 in range(0, n, bs):
        i1 = min(n, i0 + bs)
        rhs = v[..., i0:i1, :].clone()
        for j0 in range(0, i0, bs):
            j1 = min(n, j0 + bs)
            rhs -= torch.matmul(_exp_block(kh[..., i0:i1, :], kh[..., j0:j1, :], s, False), x[..., j0:j1, :])
        pii = _exp_block(kh[..., i0:i1, :], kh[..., i0:i1, :], s, True)
        x[..., i0:i1, :] = torch.linalg.solve_triangular(pii, rhs, upper=False)
        del pii, rhs
    return x


def _repeat(t: torch.Tensor, g: int) -> torch.Tensor:
    return t if g == 1 else t.repeat_interleave(g, dim=0)


def attention_fwd(q: torch.Tensor, k: torch.Tensor, x: torch.Tensor, s: float, cq: int = 4096):
    """O = softmax(s Q K^T + causal) repeat_kv(X) in query chunks of cq rows.
    Returns (o [Hq, N, D], lse [Hq, N] natural log)."""
    _no_tf32()
    hq, n, _ = q.shape
    g = hq // k.shape[0]
    kr, xr = _repeat(k, g), _repeat(x, g)
    o = torch.empty_like(q)
    lse = torch.empty(hq, n, dtype=q.dtype, device=q.device)
    for c0 in range(0, n, cq):
        c1 = min(n, c0 + cq)
        sc = torch.matmul(q[:, c0:c1], kr[:, :c1].transpose(-1, -2)).mul_(s)
        rows = torch.arange(c0, c1, device=q.device)[:, None]
        cols = torch.arange(c1, device=q.device)[None, :]
        sc.masked_fill_(cols > rows, float("-inf"))
        m = sc.amax(-1, keepdim=True)
        sc.sub_(m).exp_()
        l = sc.sum(-1, keepdim=True)
        o[:, c0:c1] = torch.matmul(sc, xr[:, :c1]) / l
        lse[:, c0:c1] = (m + l.log()).squeeze(-1)
        del sc
    return o, lse


def attention_bwd(q, k, x, o, do, lse, s: float, cq: int = 4096):
    """Gradients of sum(O * dO) for attention_fwd: (dq [Hq,N,D], dk_attn, dx [Hkv,N,D])."""
    _no_tf32()
    hq, n, d = q.shape
    hkv = k.shape[0]
    g = hq // hkv
    kr, xr = _repeat(k, g), _repeat(x, g)
    dq = torch.empty_like(q)
    dkr = torch.zeros(hq, n, d, dtype=q.dtype, device=q.device)
    dxr = torch.zeros(hq, n, d, dtype=q.dtype, device=q.device)
    for c0 in range(0, n, cq):
        c1 = min(n, c0 + cq)
        a = torch.matmul(q[:, c0:c1], kr[:, :c1].transpose(-1, -2)).mul_(s)
        rows = torch.arange(c0, c1, device=q.device)[:, None]
        cols = torch.arange(c1, device=q.device)[None, :]
        a.masked_fill_(cols > rows, float("-inf"))
        a.sub_(lse[:, c0:c1, None]).exp_()
        doc = do[:, c0:c1]
        dxr[:, :c1] += torch.matmul(a.transpose(-1, -2), doc)
        delta = (doc * o[:, c0:c1]).sum(-1, keepdim=True)
        da = torch.matmul(doc, xr[:, :c1].transpose(-1, -2))
        da.sub_(delta).mul_(a)
        del a
        dq[:, c0:c1] = s * torch.matmul(da, kr[:, :c1])
        dkr[:, :c1] += s * torch.matmul(da.transpose(-1, -2), q[:, c0:c1])
        del da
    dk = dkr.view(hkv, g, n, d).sum(1)
    dx = dxr.view(hkv, g, n, d).sum(1)
    return dq, dk, dx


def solve_bwd(kh: torch.Tensor, x: torch.Tensor, dx: torch.Tensor, s: float, bs: int):
    """(dK^, dV) of sum(X * dX) through X = P(K^)^-1 V, by blocks of bs rows:
    dV = P^-T dX (block back substitution, modeling_lucid.py:328-334) and
    dK^ = sum over block pairs i >= j of dG_ij K^_j + dG_ij^T K^_i with
    dG_ij = -s E_ij o (dV_i X_j^T) (tril on the diagonal blocks, :352-379)."""
    _no_tf32()
    n = kh.shape[-2]
    starts = list(range(0, n, bs))
    sl = [slice(i0, min(n, i0 + bs)) for i0 in starts]
    dv = torch.empty_like(dx)
    for bi in range(len(sl) - 1, -1, -1):
        i = sl[bi]
        rhs = dx[..., i, :].clone()
        for bj in range(bi + 1, len(sl)):
            j = sl[bj]
            rhs -= torch.matmul(_exp_block(kh[..., j, :], kh[..., i, :], s, False).transpose(-1, -2), dv[..., j, :])
        pii = _exp_block(kh[..., i, :], kh[..., i, :], s, True)
        dv[..., i, :] = torch.linalg.solve_triangular(pii.transpose(-1, -2), rhs, upper=True)
        del pii, rhs
    dkh = torch.zeros_like(kh)
    for bi in range(len(sl)):
        i = sl[bi]
        for bj in range(bi + 1):
            j = sl[bj]
            dg = _exp_block(kh[..., i, :], kh[..., j, :], s, bi == bj)
            dg.mul_(torch.matmul(dv[..., i, :], x[..., j, :].transpose(-1, -2))).mul_(-s)
            dkh[..., i, :] += torch.matmul(dg, kh[..., j, :])
            dkh[..., j, :] += torch.matmul(dg.transpose(-1, -2), kh[..., i, :])
            del dg
    return dkh, dv


def lucid_fwd_bwd(q, k, v, do, scale: float | None = None, eps: float = 1e-5, bs: int | None = None,
                  cq: int = 4096, backward: bool = True):
    """One LUCID layer forward (+ backward with upstream gradient do) in float32.
    q [Hq,N,D], k, v [Hkv,N,D], do [Hq,N,D].  Returns a dict with o [Hq,N,D], x and,
    with backward, dq, dk, dv."""
    n, d = k.shape[-2], k.shape[-1]
    s = d ** -0.5 if scale is None else scale
    bs = reference_block_size(n) if bs is None else bs
    kh, r = rms_norm(k, eps)
    x = solve_fwd(kh, v, s, bs)
    o, lse = attention_fwd(q, k, x, s, cq)
    out = dict(o=o, x=x)
    if not backward:
        return out
    dq, dk_attn, dx = attention_bwd(q, k, x, o, do, lse, s, cq)
    dkh, dv = solve_bwd(kh, x, dx, s, bs)
    proj = (kh * dkh).sum(-1, keepdim=True) / d
    out.update(dq=dq, dk=dk_attn + r * (dkh - proj * kh), dv=dv)
    return out
