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
