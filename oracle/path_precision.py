"""Precision models of the reference LUCID-Path forward and PaTH attention
forward — TEST INFRASTRUCTURE ONLY.

The reference's own bf16 deviation cannot be measured by running it here
(its Triton kernels return NaN in bf16 under the CPU interpreter, and the
reference is not present on the GPU machine).  This module restates
triangular_solve_fwd_kernel (lucid_path/triton_code/triangular_solve_fwd.py:99-225)
with the reference's rounding points, so that a test can compare the B200
kernels' deviation from the float64 oracle with the reference's:

  * every tensor the reference stores or casts to the input dtype is rounded
    to bf16: T_inv (solve_tril output_dtype=w.dtype, parallel.py:47-51),
    w*beta (:119), tril(q w^T) (:122), qw T_inv (:125), stril(w_beta k^T) (:128),
    w2 (:141), T_inv wbk (:146), k_new (:148) and o (:225);
  * tl.dot on float32 operands runs in TF32 on the GPU (Triton's default
    input precision): operands rounded to 10 mantissa bits (:193, :205, :208-209);
  * everything else in float32 (A_diag :131, q_new :134, exp :202/:218,
    mini_triangular_solve :221).

Block size 64 as in the reference (parallel.py:37).
"""
from __future__ import annotations

import numpy as np

__all__ = ["reference_bf16_forward", "reference_bf16_attention", "reference_bf16_k_cache"]


def _bf16(x):
    x = np.asarray(x, dtype=np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    b = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return b.astype(np.uint32).view(np.float32)


def _tf32(x):
    x = np.asarray(x, dtype=np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    b = ((b + 0x1000) >> 13) << 13          # round to nearest (ties away), 10-bit mantissa
    return b.astype(np.uint32).view(np.float32)


def _dot(a, b):
    return (a.astype(np.float64) @ b.astype(np.float64)).astype(np.float32)


def reference_bf16_forward(k, v, w, beta, q=None, scale=None, bt=64):
    """o [B, T, HQ, V] as the reference computes it from bf16 inputs."""
    q = k if q is None else q
    B, T, HQ, K = q.shape
    H = k.shape[2]
    G = HQ // H
    s = np.float32(K ** -0.5 if scale is None else scale)
    nt = (T + bt - 1) // bt
    o = np.zeros((B, T, HQ, v.shape[-1]), dtype=np.float32)
    for b in range(B):
        for hq in range(HQ):
            h = hq // G
            qn_f32, kn, w2, ld, vv, wv = [], [], [], [], [], []
            for i in range(nt):
                sl = slice(i * bt, min(T, (i + 1) * bt))
                n = sl.stop - sl.start
                bq = q[b, sl, hq].astype(np.float32)
                bk = k[b, sl, h].astype(np.float32)
                bw = w[b, sl, h].astype(np.float32)
                bb = beta[b, sl, h].astype(np.float32)
                # T_inv = (I + diag(beta) stril(W W^T))^-1 in fp32, stored bf16
                A = np.tril(_dot(bw, bw.T), -1) * bb[:, None]
                Tm = _bf16(np.linalg.inv(np.eye(n) + A.astype(np.float64)))
                wb = _bf16(bw * bb[:, None])
                qw = _bf16(np.tril(_dot(bq, bw.T)))
                qwT = _bf16(_dot(qw, Tm))
                wbk = _bf16(np.tril(_dot(wb, bk.T), -1))
                Ad = np.tril(_dot(bq, bk.T) - _dot(qwT, wbk))
                qn_f32.append(bq - _dot(qwT, wb))
                w2.append(_bf16(_dot(Tm, wb)))
                kn.append(_bf16(bk - _dot(_bf16(_dot(Tm, wbk)).T, bw)))
                ld.append(np.tril(np.exp(Ad * s - np.float32(1.0) / s), -1).astype(np.float32))
                vv.append(v[b, sl, h].astype(np.float32))
                wv.append(bw)
            O = []
            for i in range(nt):
                R = vv[i].copy()
                qt = qn_f32[i].copy()
                for j in range(i - 1, -1, -1):
                    Aij = _dot(_tf32(qt), kn[j].T)
                    Lij = np.exp(Aij * s - np.float32(1.0) / s).astype(np.float32)
                    R = R - _dot(_tf32(Lij), O[j])
                    s2 = _dot(_tf32(qt), wv[j].T)
                    qt = qt - _dot(_tf32(s2), w2[j])
                X = R.copy()
                Ld = ld[i]
                for r in range(1, X.shape[0]):
                    X[r] = X[r] - (Ld[r, :r].astype(np.float64) @ X[:r].astype(np.float64)).astype(np.float32)
                O.append(_bf16(X))
                o[b, i * bt:i * bt + X.shape[0], hq] = O[-1]
    return o


def reference_bf16_attention(k, v, w, beta, q=None, scale=None, bt=64):
    """o [B, T, HQ, V] of the reference's PaTH softmax attention forward from bf16
    inputs: intra_chunk_preprocess_fwd.py:71-121 (diagonal blocks: A from bf16
    dots, q_new / k_new / w2 stored bf16) then parallel_path_fwd.py:87-124
    (off-diagonal blocks: tl.dot(q.to(bf16), k) :91, p.to(bf16) @ v :104,
    tl.dot(q.to(bf16), w1) and s2.to(bf16) @ w2 for the query chain :105-106,
    with the query itself kept in fp32 :37-38)."""
    q = k if q is None else q
    B, T, HQ, K = q.shape
    H = k.shape[2]
    G = HQ // H
    s = np.float32(K ** -0.5 if scale is None else scale)
    sm = np.float32(s * 1.44269504)
    nt = (T + bt - 1) // bt
    o = np.zeros((B, T, HQ, v.shape[-1]), dtype=np.float32)
    for b in range(B):
        for hq in range(HQ):
            h = hq // G
            qn, kn, w2, wv, vv, od, ld, md = [], [], [], [], [], [], [], []
            for i in range(nt):
                sl = slice(i * bt, min(T, (i + 1) * bt))
                n = sl.stop - sl.start
                bq = q[b, sl, hq].astype(np.float32)
                bk = k[b, sl, h].astype(np.float32)
                bw = w[b, sl, h].astype(np.float32)
                bb = beta[b, sl, h].astype(np.float32)
                A = np.tril(_dot(bw, bw.T), -1) * bb[:, None]
                Tm = _bf16(np.linalg.inv(np.eye(n) + A.astype(np.float64)))
                wb = _bf16(bw * bb[:, None])
                qw = _bf16(np.tril(_dot(bq, bw.T)))
                qwT = _bf16(_dot(qw, Tm))
                wbk = _bf16(np.tril(_dot(wb, bk.T), -1))
                Ad = _dot(bq, bk.T) - _dot(qwT, wbk)
                z = np.where(np.tril(np.ones((n, n), dtype=bool)), Ad * sm, -np.inf).astype(np.float32)
                m = z.max(axis=1)
                pz = np.exp2(z - m[:, None]).astype(np.float32)
                od.append(_dot(_bf16(pz), v[b, sl, h].astype(np.float32)))   # p.to(bf16) @ v (:115)
                ld.append(pz.sum(axis=1))
                md.append(m)
                qn.append(bq - _dot(qwT, wb))
                w2.append(_bf16(_dot(Tm, wb)))
                kn.append(_bf16(bk - _dot(_bf16(_dot(Tm, wbk)).T, bw)))
                wv.append(bw)
                vv.append(v[b, sl, h].astype(np.float32))
            for i in range(nt):
                bq = qn[i].copy()
                bo, bl, bm = od[i].copy(), ld[i].copy(), md[i].copy()
                for j in range(i - 1, -1, -1):
                    z = _dot(_bf16(bq), kn[j].T) * sm
                    mn = np.maximum(bm, z.max(axis=1))
                    alpha = np.exp2(bm - mn)
                    pz = np.exp2(z - mn[:, None]).astype(np.float32)
                    bo = bo * alpha[:, None]
                    bl = bl * alpha + pz.sum(axis=1)
                    bm = mn
                    bo = bo + _dot(_bf16(pz), vv[j])
                    s2 = _dot(_bf16(bq), wv[j].T)
                    bq = bq - _dot(_bf16(s2), w2[j])
                o[b, i * bt:i * bt + bo.shape[0], hq] = _bf16(bo / bl[:, None])
    return o


def reference_bf16_k_cache(k, w, beta, bt=64):
    """k_cache [B, T, H, K] of use_cache=True as the reference computes it:
    k_new and w2 from triangular_solve_fwd (stored bf16, :141-148), then
    prepare_k_cache.py:36-47 with the key in fp32 and the products on bf16
    operands (b_k.to(w2.dtype), b_A.to(w1.dtype)), stored bf16."""
    B, T, H, K = k.shape
    nt = (T + bt - 1) // bt
    out = np.zeros(k.shape, dtype=np.float32)
    for b in range(B):
        for h in range(H):
            kn, w2, wv = [], [], []
            for i in range(nt):
                sl = slice(i * bt, min(T, (i + 1) * bt))
                n = sl.stop - sl.start
                bk = k[b, sl, h].astype(np.float32)
                bw = w[b, sl, h].astype(np.float32)
                bb = beta[b, sl, h].astype(np.float32)
                A = np.tril(_dot(bw, bw.T), -1) * bb[:, None]
                Tm = _bf16(np.linalg.inv(np.eye(n) + A.astype(np.float64)))
                wb = _bf16(bw * bb[:, None])
                wbk = _bf16(np.tril(_dot(wb, bk.T), -1))
                w2.append(_bf16(_dot(Tm, wb)))
                kn.append(_bf16(bk - _dot(_bf16(_dot(Tm, wbk)).T, bw)))
                wv.append(bw)
            for i in range(nt):
                bk = kn[i].copy()
                for j in range(i + 1, nt):
                    bA = _dot(_bf16(bk), w2[j].T)
                    bk = bk - _dot(_bf16(bA), wv[j])
                out[b, i * bt:i * bt + bk.shape[0], h] = _bf16(bk)
    return out
