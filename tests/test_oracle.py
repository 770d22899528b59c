"""The CPU oracle (oracle/lucid_oracle.py) against the reference's own
outputs (tests/golden/*.npz, produced by tests/golden/make_golden.py from
modeling_lucid.py).  CPU only."""
import numpy as np
import pytest

from conftest import DECODE_CASES, load_decode_golden, ATTN_CASES, load_golden
from oracle import lucid_oracle as orc


def _close(a, b, rtol=1e-5):
    scale = max(1.0, float(np.max(np.abs(b))))
    np.testing.assert_allclose(a, b, rtol=0, atol=rtol * scale)


@pytest.mark.parametrize("case", ATTN_CASES)
def test_oracle_forward_matches_reference(case):
    g = load_golden(case)
    o, x = orc.lucid_fwd(g["q"], g["k"], g["v"], float(g["scale"]), float(g["eps"]))
    _close(x, g["x"])
    _close(o, g["o"])


@pytest.mark.parametrize("case", ATTN_CASES)
def test_oracle_backward_matches_reference(case):
    g = load_golden(case)
    dq, dk, dv = orc.lucid_bwd(g["q"], g["k"], g["v"], g["do"], float(g["scale"]), float(g["eps"]))
    _close(dq, g["dq"])
    _close(dk, g["dk"])
    _close(dv, g["dv"])


def test_oracle_blockwise_matches_reference_solver():
    """Lucid_Tril_Solver (modeling_lucid.py:284-382) with BS=16."""
    g = load_golden("blockwise_bs16")
    scale = float(g["scale"])
    x_blk = orc.blockwise_solve(g["khat"], g["v"], scale, int(g["bs"]))
    x_dense = np.linalg.solve(orc.p_from_khat(g["khat"], scale), g["v"])
    _close(x_blk, g["x"], 1e-9)
    _close(x_dense, g["x"], 1e-9)


def test_oracle_blockwise_backward_matches_reference_solver():
    g = load_golden("blockwise_bs16")
    scale = float(g["scale"])
    dkh, dv = orc.blockwise_solve_bwd(g["khat"], g["x"], g["dx"], scale)
    _close(dv, g["dv"], 1e-9)
    _close(dkh, g["dkhat"], 1e-9)


def test_oracle_gradient_finite_difference():
    """Directional derivative of sum(O * dO) vs the analytic backward."""
    rng = np.random.default_rng(0)
    B, Hq, Hkv, N, D = 1, 2, 1, 20, 8
    q = rng.standard_normal((B, Hq, N, D))
    k = rng.standard_normal((B, Hkv, N, D))
    v = rng.standard_normal((B, Hkv, N, D))
    do = rng.standard_normal((B, N, Hq, D))
    s = D ** -0.5
    dq, dk, dv = orc.lucid_bwd(q, k, v, do, s)
    f = lambda q_, k_, v_: float(np.sum(orc.lucid_fwd(q_, k_, v_, s)[0] * do))
    h = 1e-6
    for grad, which in ((dq, 0), (dk, 1), (dv, 2)):
        dirn = rng.standard_normal(grad.shape)
        args_p = [q, k, v]
        args_m = [q, k, v]
        args_p[which] = args_p[which] + h * dirn
        args_m[which] = args_m[which] - h * dirn
        fd = (f(*args_p) - f(*args_m)) / (2 * h)
        assert abs(fd - float(np.sum(grad * dirn))) < 1e-5 * max(1.0, abs(fd))


def test_oracle_stress_conditioning():
    """The correlated-key distribution of the long-context config gives a
    well-posed but non-trivial P (off-diagonal mass of order 1)."""
    g = load_golden("stress_d128")
    p = orc.build_p(g["k"], float(g["scale"]), float(g["eps"]))[0, 0]
    off = p - np.diag(np.diag(p))
    assert np.all(np.isfinite(p))
    assert off.sum(axis=1).max() > 0.05
    assert np.all(np.abs(np.diag(p) - 1.0) < 1e-3)


@pytest.mark.parametrize("name", DECODE_CASES)
def test_decode_oracle_matches_reference_fixture(name):
    """get_new_v_prime (modeling_lucid.py:576-598) of the reference against the oracle."""
    from oracle.lucid_oracle import decode_update
    d = load_decode_golden(name)
    x = decode_update(d["k_new"], d["v_new"], d["k_cache"], d["x_cache"], float(d["scale"]), float(d["eps"]))
    assert np.max(np.abs(x - d["x_new"])) < 1e-5
