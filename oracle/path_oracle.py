"""CPU oracle for LUCID-Path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may import this module, and only as the checker or the timed CPU
baseline.  The product path (lucid_b200) never calls it.

Float64 numpy restatement of the reference's LUCID-Path op
(saisuryadv/LUCID, lucid_path/triton_code/):

  H_t  = I - beta_t w_t w_t^T                      (Householder, beta in (0, 2))
  A_rc = q_r^T (H_r H_{r-1} ... H_{c+1}) k_c, r > c (triangular_solve_fwd.py:118-148 diagonal
                                                     blocks via the UT transform, :177-209 the
                                                     off-diagonal blocks with the progressive
                                                     q update q <- q - (q w_j^T) w2_j)
  L    = stril(exp(s A - 1/s))                      (:202, :218)
  O    = (I + L)^-1 V                               (:221, mini_tril_solve.py:42-61; unit diagonal)

Layouts follow parallel.py:180-241: k, v, w [B, T, H, K]; beta [B, T, H];
q [B, T, HQ, K] (defaults to k); o [B, T, HQ, V]; v is shared by the G = HQ/H
query heads of a key head (triangular_solve_fwd.py:53, :85-86).

Two restatements are given:

* ``path_fwd`` — the dense definition above (explicit Householder products).
* ``path_fwd_blockwise`` / ``path_bwd_blockwise`` — the block decomposition
  the sm_100a kernels implement (UT transform per block, descending query
  chain for the off-diagonal scores, wavefront solve; backward: transposed
  solve, ascending dQ~ chain, column sums dK_new / Phi, per-block prep
  backward).  They are checked against ``path_fwd`` and against float64
  autograd (``path_fwd_bwd_torch``) by tests/test_path_oracle.py, and the
  dense definition is pinned to the reference Triton op by the fixtures of
  tests/golden/make_path_golden.py.
"""
from __future__ import annotations

import numpy as np

__all__ = ["path_scores", "path_fwd", "path_fwd_blockwise", "path_bwd_blockwise", "path_fwd_bwd_torch",
           "make_path_inputs", "path_attention_fwd", "path_k_cache"]


def make_path_inputs(seed: int, B: int, T: int, H: int, K: int, HQ: int | None = None, with_q: bool = False):
    """Seeded inputs with the distributions of the LUCID-Path benchmark config:
    k, v, q ~ N(0,1); w ~ N(0,1) L2-normalised per head vector; beta = 2 sigmoid(N(0,1));
    do ~ N(0,1).  Returned as float64 arrays rounded to bf16-representable values."""
    rng = np.random.default_rng(seed)
    HQ = HQ or H

    def bf(x):
        x = np.asarray(x, dtype=np.float32)
        b = x.view(np.uint32)
        b = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16  # round to nearest even
        return b.astype(np.uint32).view(np.float32).astype(np.float64)

    k = bf(rng.standard_normal((B, T, H, K)))
    v = bf(rng.standard_normal((B, T, H, K)))
    w = rng.standard_normal((B, T, H, K))
    w = bf(w / np.linalg.norm(w, axis=-1, keepdims=True))
    beta = bf(2.0 / (1.0 + np.exp(-rng.standard_normal((B, T, H)))))
    q = bf(rng.standard_normal((B, T, HQ, K))) if with_q else None
    do = bf(rng.standard_normal((B, T, HQ, K)))
    return dict(q=q, k=k, v=v, w=w, beta=beta, do=do)


def _heads(q, k):
    HQ, H = q.shape[2], k.shape[2]
    assert HQ % H == 0
    return HQ, H, HQ // H


def path_scores(q, k, w, beta):
    """A[b, hq, r, c] = q_r^T (H_r ... H_{c+1}) k_c for r > c, 0 elsewhere.

    Keys are carried forward: after step r every key c < r holds
    (H_r ... H_{c+1}) k_c, so row r of A is a matrix-vector product."""
    B, T, HQ, K = q.shape
    _, H, G = _heads(q, k)
    A = np.zeros((B, HQ, T, T))
    for b in range(B):
        for hq in range(HQ):
            h = hq // G
            X = k[b, :, h, :].copy()
            for r in range(1, T):
                wr = w[b, r, h]
                X[:r] -= beta[b, r, h] * np.outer(X[:r] @ wr, wr)
                A[b, hq, r, :r] = X[:r] @ q[b, r, hq]
    return A


def path_k_cache(k, w, beta):
    """Decode-time keys of use_cache=True (prepare_k_cache.py:8-49): every key
    transformed by all later Householders, k_cache_c = (H_{T-1} ... H_{c+1}) k_c."""
    B, T, H, K = k.shape
    out = np.zeros_like(k)
    for b in range(B):
        for h in range(H):
            X = k[b, :, h, :].copy()
            for r in range(1, T):
                wr = w[b, r, h]
                X[:r] -= beta[b, r, h] * np.outer(X[:r] @ wr, wr)
            out[b, :, h] = X
    return out


def path_attention_fwd(k, v, w, beta, q=None, scale=None):
    """PaTH softmax attention forward (parallel_path_fwd.py:13-124 with the diagonal
    blocks of intra_chunk_preprocess_fwd.py:13-121):
        O_r = sum_{c <= r} softmax_c(s A_rc) v_c,  A_rc = q_r^T (H_r ... H_{c+1}) k_c
    (A_rr = q_r . k_r).  Returns (o [B,T,HQ,V], lse [B,T,HQ]) with lse the
    log2-sum-exp of s A log2(e) over the row, as the reference stores L_new."""
    q = k if q is None else q
    B, T, HQ, K = q.shape
    _, H, G = _heads(q, k)
    s = K ** -0.5 if scale is None else scale
    A = path_scores(q, k, w, beta)
    o = np.zeros((B, T, HQ, v.shape[-1]))
    lse = np.zeros((B, T, HQ))
    for b in range(B):
        for hq in range(HQ):
            h = hq // G
            Ab = A[b, hq].copy()
            Ab[np.arange(T), np.arange(T)] = np.einsum("td,td->t", q[b, :, hq], k[b, :, h])
            z = np.where(np.tril(np.ones((T, T), dtype=bool)), s * Ab * np.log2(np.e), -np.inf)
            m = z.max(axis=1, keepdims=True)
            p = np.exp2(z - m)
            l = p.sum(axis=1, keepdims=True)
            o[b, :, hq] = (p / l) @ v[b, :, h]
            lse[b, :, hq] = (np.log2(l) + m)[:, 0]
    return o, lse


def _unit_lower_solve(L, R):
    """(I + L) X = R for strictly-lower L (forward substitution, mini_tril_solve.py:42-61)."""
    X = R.copy()
    for i in range(1, L.shape[0]):
        X[i] -= L[i, :i] @ X[:i]
    return X


def _unit_upper_solve_t(L, R):
    """(I + L)^T X = R for strictly-lower L (backward substitution, mini_tril_solve.py:62-79)."""
    X = R.copy()
    n = L.shape[0]
    for i in range(n - 2, -1, -1):
        X[i] -= L[i + 1:, i] @ X[i + 1:]
    return X


def path_fwd(k, v, w, beta, q=None, scale=None):
    """Dense definition; returns (o [B,T,HQ,V], L [B,HQ,T,T])."""
    q = k if q is None else q
    B, T, HQ, K = q.shape
    _, H, G = _heads(q, k)
    s = K ** -0.5 if scale is None else scale
    A = path_scores(q, k, w, beta)
    L = np.tril(np.exp(s * A - 1.0 / s), -1)
    o = np.zeros((B, T, HQ, v.shape[-1]))
    for b in range(B):
        for hq in range(HQ):
            o[b, :, hq] = _unit_lower_solve(L[b, hq], v[b, :, hq // G])
    return o, L


# --------------------------------------------------------------------------------------------
# Block decomposition (what the kernels compute), float64.
# --------------------------------------------------------------------------------------------

def _prep_block(Qb, Kb, Wb, bb, s):
    """Per-block quantities (triangular_solve_fwd.py:118-148, UT transform of parallel.py:39-51):
    T = (I + stril(diag(beta) W W^T))^-1, W2 = T diag(beta) W, Q_new = Q - tril(Q W^T) W2,
    K_new = K - (T stril(diag(beta) W K^T))^T W, A_diag = tril(Q K^T - tril(Q W^T) T stril(diag(beta) W K^T)),
    L_diag = stril(exp(s A_diag - 1/s))."""
    n = Qb.shape[0]
    Wb_beta = bb[:, None] * Wb
    M = np.tril(Wb_beta @ Wb.T, -1)
    Tm = np.linalg.inv(np.eye(n) + M)
    W2 = Tm @ Wb_beta
    QW = np.tril(Qb @ Wb.T)
    Qn = Qb - QW @ W2
    WbK = np.tril(Wb_beta @ Kb.T, -1)
    TB = Tm @ WbK
    Kn = Kb - TB.T @ Wb
    Ad = np.tril(Qb @ Kb.T - QW @ TB)
    Ld = np.tril(np.exp(s * Ad - 1.0 / s), -1)
    return dict(T=Tm, W2=W2, QW=QW, Qn=Qn, WbK=WbK, TB=TB, Kn=Kn, Ld=Ld, Wb_beta=Wb_beta)


def _blocks(T, bt):
    nb = (T + bt - 1) // bt
    return nb, [slice(i * bt, min(T, (i + 1) * bt)) for i in range(nb)]


def path_fwd_blockwise(k, v, w, beta, q=None, scale=None, bt=128):
    """Forward of the kernels: per block prep, descending query chain for L_ij (i > j),
    then the block forward substitution.  Returns (o, state) where state holds
    every intermediate the backward reuses (per b, hq)."""
    q = k if q is None else q
    B, T, HQ, K = q.shape
    _, H, G = _heads(q, k)
    s = K ** -0.5 if scale is None else scale
    nb, sl = _blocks(T, bt)
    o = np.zeros((B, T, HQ, v.shape[-1]))
    state = {}
    for b in range(B):
        for hq in range(HQ):
            h = hq // G
            P = [_prep_block(q[b, sl[i], hq], k[b, sl[i], h], w[b, sl[i], h], beta[b, sl[i], h], s)
                 for i in range(nb)]
            Lt, Qs = {}, {}
            for i in range(nb):
                qt = P[i]["Qn"].copy()                      # Q~_i^{(i-1)}
                for j in range(i - 1, -1, -1):
                    Qs[i, j] = qt.copy()
                    Lt[i, j] = np.exp(s * (qt @ P[j]["Kn"].T) - 1.0 / s)
                    qt = qt - (qt @ w[b, sl[j], h].T) @ P[j]["W2"]
                Lt[i, i] = P[i]["Ld"]
            X = [None] * nb
            for i in range(nb):
                R = v[b, sl[i], h].copy()
                for j in range(i):
                    R -= Lt[i, j] @ X[j]
                X[i] = _unit_lower_solve(Lt[i, i], R)
                o[b, sl[i], hq] = X[i]
            state[b, hq] = dict(P=P, L=Lt, Qs=Qs, X=X)
    return o, state


def _prep_block_bwd(Qb, Kb, Wb, bb, pr, dA, dQn, dKn, dW2, dW_in, s):
    """Backward of _prep_block for one query head (dA strictly lower), returning
    (dQ, dK, dW, dbeta).  Every step mirrors one line of the forward."""
    Wb_beta, Tm, W2, QW, TB, WbK = pr["Wb_beta"], pr["T"], pr["W2"], pr["QW"], pr["TB"], pr["WbK"]
    dQ = np.zeros_like(Qb); dK = np.zeros_like(Kb); dW = dW_in.copy(); dWb = np.zeros_like(Wb)
    dTB = np.zeros_like(TB); dT = np.zeros_like(Tm); dQW = np.zeros_like(QW); dW2 = dW2.copy()
    # A = tril(Q K^T - QW TB)
    dQ += dA @ Kb; dK += dA.T @ Qb; dQW -= dA @ TB.T; dTB -= QW.T @ dA
    # Q_new = Q - QW W2
    dQ += dQn; dQW -= dQn @ W2.T; dW2 -= QW.T @ dQn
    # QW = tril(Q W^T)
    dQW = np.tril(dQW); dQ += dQW @ Wb; dW += dQW.T @ Qb
    # K_new = K - TB^T W
    dK += dKn; dTB -= Wb @ dKn.T; dW -= TB @ dKn
    # TB = T WbK
    dT += dTB @ WbK.T; dWbK = np.tril(Tm.T @ dTB, -1)
    # WbK = stril(Wb_beta K^T)
    dWb += dWbK @ Kb; dK += dWbK.T @ Wb_beta
    # W2 = T Wb_beta
    dT += dW2 @ Wb_beta.T; dWb += Tm.T @ dW2
    # T = (I + M)^-1,  M = stril(Wb_beta W^T)
    dM = np.tril(-Tm.T @ dT @ Tm.T, -1)
    dWb += dM @ Wb; dW += dM.T @ Wb_beta
    # Wb_beta = diag(beta) W
    dbeta = np.sum(dWb * Wb, axis=1); dW += bb[:, None] * dWb
    return dQ, dK, dW, dbeta


def path_bwd_blockwise(k, v, w, beta, do, q=None, scale=None, bt=128):
    """Backward of the kernels' decomposition.  Returns (dq, dk, dv, dw, dbeta)
    with q's gradient folded into dk when q is None (q = k, parallel.py:224-225).

      dV_hq  = (I + L)^-T dO                             transposed block solve
      dA_ij  = -s L_ij o (dV_i O_j^T)                    every block pair j <= i (strictly lower)
      row i  : dQ~^{(j)} = dQ~^{(j-1)} G_j^T + dA_ij K_new_j,  j = 0 .. i-1,  G_j = I - W_j^T W2_j
               dQ_new_i = dQ~^{(i-1)}
      col j  : dK_new_j = sum_{i>j} dA_ij^T Q~_i^{(j)}
               Phi_j    = sum_{i>j} Q~_i^{(j)T} dQ~_i^{(j-1)}   (gradient of G_j)
               dW2_j   -= W_j Phi_j,   dW_j -= W2_j Phi_j^T
      block  : _prep_block_bwd with dA_ii, dQ_new, dK_new, dW2, dW
    """
    q_given = q is not None
    q = k if q is None else q
    B, T, HQ, K = q.shape
    _, H, G = _heads(q, k)
    s = K ** -0.5 if scale is None else scale
    o, st = path_fwd_blockwise(k, v, w, beta, q=q, scale=s, bt=bt)
    nb, sl = _blocks(T, bt)
    dq = np.zeros_like(q); dk = np.zeros_like(k); dv = np.zeros_like(v)
    dw = np.zeros_like(w); dbeta = np.zeros_like(beta)
    for b in range(B):
        for hq in range(HQ):
            h = hq // G
            S = st[b, hq]; P, Lt, Qs, X = S["P"], S["L"], S["Qs"], S["X"]
            Wj = [w[b, sl[j], h] for j in range(nb)]
            # transposed solve
            dV = [None] * nb
            for j in range(nb - 1, -1, -1):
                R = do[b, sl[j], hq].copy()
                for i in range(j + 1, nb):
                    R -= Lt[i, j].T @ dV[i]
                dV[j] = _unit_upper_solve_t(Lt[j, j], R)
                dv[b, sl[j], h] += dV[j]
            dA = {}
            for i in range(nb):
                for j in range(i + 1):
                    d = -s * Lt[i, j] * (dV[i] @ X[j].T)
                    dA[i, j] = np.tril(d, -1) if i == j else d
            # row pass
            dQn, Dq = [None] * nb, {}
            for i in range(nb):
                g = np.zeros((sl[i].stop - sl[i].start, K))
                for j in range(i):
                    Dq[i, j] = g.copy()                      # dQ~_i^{(j-1)}
                    g = g - (g @ P[j]["W2"].T) @ Wj[j] + dA[i, j] @ P[j]["Kn"]
                dQn[i] = g
            # column pass
            dKn, dW2, dWi = [None] * nb, [None] * nb, [None] * nb
            for j in range(nb):
                acc = np.zeros_like(P[j]["Kn"]); phi = np.zeros((K, K))
                for i in range(j + 1, nb):
                    acc += dA[i, j].T @ Qs[i, j]
                    phi += Qs[i, j].T @ Dq[i, j]
                dKn[j] = acc
                dW2[j] = -Wj[j] @ phi
                dWi[j] = -P[j]["W2"] @ phi.T
            for i in range(nb):
                dQb, dKb, dWb, dbb = _prep_block_bwd(q[b, sl[i], hq], k[b, sl[i], h], Wj[i], beta[b, sl[i], h],
                                                     P[i], dA[i, i], dQn[i], dKn[i], dW2[i], dWi[i], s)
                dq[b, sl[i], hq] += dQb
                dk[b, sl[i], h] += dKb
                dw[b, sl[i], h] += dWb
                dbeta[b, sl[i], h] += dbb
    if not q_given:
        dk = dk + dq
        dq = None
    return dq, dk, dv, dw, dbeta


# --------------------------------------------------------------------------------------------
# float64 autograd of the dense definition (checker for the analytic backward above).
# --------------------------------------------------------------------------------------------

def path_fwd_bwd_torch(k, v, w, beta, do, q=None, scale=None):
    """Dense definition in torch float64 with autograd; returns o and the
    gradients (dq or None, dk, dv, dw, dbeta) exactly as the reference
    op hands them to autograd (q = k folds dq into dk)."""
    import torch
    t = lambda a: torch.tensor(a, dtype=torch.float64, requires_grad=True)
    kt, vt, wt, bt_ = t(k), t(v), t(w), t(beta)
    qt = t(q) if q is not None else kt
    B, T, HQ, K = qt.shape
    H = kt.shape[2]; G = HQ // H
    s = K ** -0.5 if scale is None else scale
    outs = []
    for b in range(B):
        per_h = []
        for hq in range(HQ):
            h = hq // G
            X = kt[b, :, h, :]
            rows = [torch.zeros(T, dtype=torch.float64)]
            for r in range(1, T):
                wr = wt[b, r, h]
                upd = bt_[b, r, h] * torch.outer(X[:r] @ wr, wr)
                X = torch.cat([X[:r] - upd, X[r:]], 0)
                a = X[:r] @ qt[b, r, hq]
                rows.append(torch.cat([a, torch.zeros(T - r, dtype=torch.float64)]))
            A = torch.stack(rows)
            L = torch.tril(torch.exp(s * A - 1.0 / s), -1)
            P = torch.eye(T, dtype=torch.float64) + L
            per_h.append(torch.linalg.solve_triangular(P, vt[b, :, h, :], upper=False, unitriangular=True))
        outs.append(torch.stack(per_h, 1))
    o = torch.stack(outs, 0)
    o.backward(torch.tensor(do, dtype=torch.float64))
    dq = qt.grad.numpy() if q is not None else None
    return o.detach().numpy(), dq, kt.grad.numpy(), vt.grad.numpy(), wt.grad.numpy(), bt_.grad.numpy()
