"""The torch CPU restatement used as the timed CPU baseline
(oracle/torch_ref.py) reproduces the reference's outputs (golden fixtures)."""
import numpy as np
import pytest
import torch

from conftest import ATTN_CASES, load_golden
from oracle import torch_ref


@pytest.mark.parametrize("case", ATTN_CASES)
def test_torch_port_matches_reference(case):
    g = load_golden(case)
    t = lambda a: torch.as_tensor(a, dtype=torch.float64)
    o, dq, dk, dv = torch_ref.lucid_fwd_bwd(t(g["q"]), t(g["k"]), t(g["v"]), t(g["do"]),
                                            float(g["scale"]), float(g["eps"]))
    for got, want in ((o, g["o"]), (dq, g["dq"]), (dk, g["dk"]), (dv, g["dv"])):
        np.testing.assert_allclose(got.numpy(), want, atol=1e-5 * max(1.0, np.abs(want).max()))


@pytest.mark.parametrize("hq,hkv,n,bs,keys", [(2, 2, 200, 200, "iid"), (2, 2, 200, 64, "corr"),
                                              (4, 2, 150, 48, "iid"), (1, 1, 97, 32, "corr")])
def test_torch_blockwise_matches_oracle(hq, hkv, n, bs, keys):
    """The float32 full-length reference (oracle/torch_blockwise.py: dense branch with one
    block, Lucid_Tril_Solver's row blocks otherwise, chunked attention, analytic backward)
    against the float64 oracle, here in float64."""
    from oracle import lucid_oracle as orc
    from oracle import torch_blockwise as tb
    rng = np.random.default_rng(n + bs)
    d = 32
    q = rng.standard_normal((1, hq, n, d))
    if keys == "iid":
        k = rng.standard_normal((1, hkv, n, d))
    else:
        k = 0.6 * rng.standard_normal((1, hkv, 1, d)) + 0.8 * rng.standard_normal((1, hkv, n, d))
    v = rng.standard_normal((1, hkv, n, d))
    do = rng.standard_normal((1, n, hq, d))
    s = d ** -0.5
    o_r, dq_r, dk_r, dv_r = orc.lucid_fwd_bwd(q, k, v, do, s)
    x_r = orc.solve(k, v, s, 1e-5)
    t = lambda a: torch.as_tensor(a[0], dtype=torch.float64)
    out = tb.lucid_fwd_bwd(t(q), t(k), t(v), torch.as_tensor(np.swapaxes(do, 1, 2)[0]), s, bs=bs, cq=40)
    for got, want in ((out["x"], x_r[0]), (out["o"], np.swapaxes(o_r, 1, 2)[0]), (out["dq"], dq_r[0]),
                      (out["dk"], dk_r[0]), (out["dv"], dv_r[0])):
        np.testing.assert_allclose(got.numpy(), want, atol=1e-9 * max(1.0, np.abs(want).max()))


def test_reference_block_size():
    from oracle import torch_blockwise as tb
    assert tb.reference_block_size(32768) == 32768
    assert tb.reference_block_size(65536) == 2 ** 14
    assert tb.reference_block_size(131072) == 2 ** 14
