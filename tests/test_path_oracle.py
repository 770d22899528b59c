"""The LUCID-Path oracle (oracle/path_oracle.py) against the reference.

The fixtures were produced by the reference's own Triton op
(lucid_path/triton_code/parallel.py) in float32 under the Triton CPU
interpreter; the oracle is float64, so agreement is to float32 rounding.
The block decomposition the kernels implement is checked against the dense
definition and against float64 autograd at several block sizes, including
ragged sequence lengths and grouped query heads."""
import numpy as np
import pytest

from conftest import PATH_ATTN_CASES, PATH_CASES, load_path_golden
from oracle.path_oracle import (make_path_inputs, path_attention_fwd, path_bwd_blockwise, path_fwd,
                                path_fwd_blockwise, path_fwd_bwd_torch)

GRADS = ("dq", "dk", "dv", "dw", "dbeta")


def _rel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


@pytest.mark.parametrize("name", PATH_CASES)
def test_oracle_matches_reference_fixture(name):
    d = load_path_golden(name)
    o, dq, dk, dv, dw, db = path_fwd_bwd_torch(d["k"], d["v"], d["w"], d["beta"], d["do"], q=d["q"])
    assert _rel(o, d["o"]) < 1e-6
    for nm, a in zip(GRADS, (dq, dk, dv, dw, db)):
        if a is None:
            assert nm not in d
            continue
        assert _rel(a, d[nm]) < 5e-6, nm


@pytest.mark.parametrize("name", PATH_CASES)
def test_block_decomposition_matches_reference_fixture(name):
    d = load_path_golden(name)
    bt = 128 if d["k"].shape[-1] == 128 else 64
    o, _ = path_fwd_blockwise(d["k"], d["v"], d["w"], d["beta"], q=d["q"], bt=bt)
    assert _rel(o, d["o"]) < 1e-6
    grads = path_bwd_blockwise(d["k"], d["v"], d["w"], d["beta"], d["do"], q=d["q"], bt=bt)
    for nm, a in zip(GRADS, grads):
        if a is None:
            continue
        assert _rel(a, d[nm]) < 5e-6, nm


@pytest.mark.parametrize("B,T,H,K,HQ,with_q,bt", [(1, 40, 1, 8, 1, False, 8), (2, 37, 2, 8, 4, True, 8),
                                                  (1, 64, 1, 16, 1, False, 16), (1, 5, 1, 8, 1, False, 8)])
def test_block_decomposition_is_exact(B, T, H, K, HQ, with_q, bt):
    d = make_path_inputs(7, B, T, H, K, HQ, with_q)
    o, _ = path_fwd(d["k"], d["v"], d["w"], d["beta"], q=d["q"])
    ob, _ = path_fwd_blockwise(d["k"], d["v"], d["w"], d["beta"], q=d["q"], bt=bt)
    assert np.max(np.abs(o - ob)) < 1e-12
    ref = path_fwd_bwd_torch(d["k"], d["v"], d["w"], d["beta"], d["do"], q=d["q"])
    got = path_bwd_blockwise(d["k"], d["v"], d["w"], d["beta"], d["do"], q=d["q"], bt=bt)
    for nm, a, b in zip(GRADS, ref[1:], got):
        assert (a is None) == (b is None), nm
        if a is not None:
            assert np.max(np.abs(a - b)) < 1e-11, nm


def test_unit_diagonal_and_identity_limit():
    """w = 0 makes every H_t the identity, so A = Q K^T (strictly lower) and
    the op reduces to (I + stril(exp(s QK^T - 1/s)))^-1 V."""
    d = make_path_inputs(3, 1, 24, 1, 8)
    w = np.zeros_like(d["w"])
    o, L = path_fwd(d["k"], d["v"], w, d["beta"])
    k = d["k"][0, :, 0]
    s = 8 ** -0.5
    Lr = np.tril(np.exp(s * k @ k.T - 1 / s), -1)
    assert np.allclose(L[0, 0], Lr)
    assert np.allclose(o[0, :, 0], np.linalg.solve(np.eye(24) + Lr, d["v"][0, :, 0]))


def test_reference_precision_model_is_close_to_float64():
    """The bf16/TF32 model of the reference forward stays within bf16 error of
    the float64 oracle, and equals it when every rounding point is exact
    (w = 0, integer-valued v, L tiny)."""
    from oracle.path_precision import reference_bf16_forward
    d = make_path_inputs(4, 1, 200, 1, 128)
    o, _ = path_fwd(d["k"], d["v"], d["w"], d["beta"])
    om = reference_bf16_forward(d["k"], d["v"], d["w"], d["beta"])
    assert np.abs(om - o).max() < 1e-2
    d2 = make_path_inputs(4, 1, 150, 2, 32, HQ=4, with_q=True)
    o2, _ = path_fwd(d2["k"], d2["v"], d2["w"], d2["beta"], q=d2["q"])
    om2 = reference_bf16_forward(d2["k"], d2["v"], d2["w"], d2["beta"], q=d2["q"])
    assert np.abs(om2 - o2).max() < 3e-2


@pytest.mark.parametrize("name", PATH_ATTN_CASES)
def test_path_attention_oracle_matches_reference_fixture(name):
    """PaTH softmax attention (intra_chunk_preprocess_fwd + parallel_path_fwd of the
    reference, float32 in the Triton interpreter) against the dense float64 oracle."""
    d = load_path_golden(name)
    o, lse = path_attention_fwd(d["k"], d["v"], d["w"], d["beta"], q=d["q"])
    assert _rel(o, d["o"]) < 1e-6
    assert np.max(np.abs(lse - d["lse"])) < 1e-4
