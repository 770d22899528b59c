"""GPU parity at the benchmark configurations' own shapes, against the float32 reference
the op's tolerance is defined on: the reference's training path in float32
(torch.linalg.solve_triangular for the solve, exact causal softmax attention, the
analytic backward), run on the same GPU by oracle/torch_blockwise.py on the same
bf16-exact inputs.

  config 2        B4 H32 N4096 D128, every (batch, head): O, dQ, dK, dV
  32K headline    B1 H32 N32768, the op over all heads, two heads compared
  N = 65536       one head: the reference's blockwise branch (Lucid_Tril_Solver,
                  modeling_lucid.py:285-382, row blocks of 2**14), fwd + bwd
  128K stress     one head, K = 0.6 s + 0.8 n (P's row sums reach ~11): X, O and the
                  gradients
  LUCID-Path      T = 16384, one (batch, head), against the float64 block restatement

Bars (tests/parity.py): |ours - ref| <= 1e-2 + ulp_bf16(ref)/2 (the op's max-abs 1e-2
applied before the final bf16 rounding) and the earlier 1e-2 + 2^-8 |ref|; the measured
max-abs values are listed in the terminal summary.
"""
import numpy as np
import pytest

import parity

pytestmark = pytest.mark.gpu

D = 128


def _inputs(dev, seed, B, H, N, q_scale=1.0, keys="iid"):
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g, device=dev, dtype=torch.float32)
    q = (r(B, H, N, D) * q_scale).to(torch.bfloat16)
    if keys == "iid":
        k = r(B, H, N, D)
    else:  # K = 0.6 s + 0.8 n, s shared per head (the 128K stress distribution)
        k = 0.6 * r(B, H, 1, D) + 0.8 * r(B, H, N, D)
    k = k.to(torch.bfloat16)
    v = r(B, H, N, D).to(torch.bfloat16)
    do = r(B, N, H, D).to(torch.bfloat16)
    return q, k, v, do


def _ours(q, k, v, do):
    import torch
    from lucid_b200 import lucid_attention
    qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = lucid_attention(qq, kk, vv)
    o.backward(do)
    torch.cuda.synchronize()
    return o.detach(), qq.grad, kk.grad, vv.grad


def _reference(q, k, v, do, b, hs, backward=True):
    """float32 reference for batch b, heads hs (a slice): tensors [H, N, D]."""
    from oracle import torch_blockwise as tb
    f = lambda t: t[b, hs].float()
    return tb.lucid_fwd_bwd(f(q), f(k), f(v), do[b, :, hs].transpose(0, 1).float(), backward=backward)


def _compare(case, ours, ref, b, hs):
    o, dq, dk, dv = ours
    parity.check_torch(o[b, :, hs].transpose(0, 1), ref["o"], case, "O")
    parity.check_torch(dq[b, hs], ref["dq"], case, "dQ")
    parity.check_torch(dk[b, hs], ref["dk"], case, "dK")
    parity.check_torch(dv[b, hs], ref["dv"], case, "dV")


def test_config2_full(cuda_device):
    """B4 H32 N4096 D128, Q ~ N(0,1)/sqrt(128), K, V, dO ~ N(0,1)."""
    import torch
    B, H, N = 4, 32, 4096
    q, k, v, do = _inputs(cuda_device, 2, B, H, N, q_scale=D ** -0.5)
    ours = _ours(q, k, v, do)
    refs = {n: torch.empty(B, H, N, D, dtype=torch.float32, device=cuda_device) for n in ("o", "dq", "dk", "dv")}
    for b in range(B):
        for h0 in range(0, H, 8):
            hs = slice(h0, h0 + 8)
            r = _reference(q, k, v, do, b, hs)
            for n in refs:
                refs[n][b, hs] = r[n]
            del r
    o, dq, dk, dv = ours
    parity.check_torch(o.transpose(1, 2), refs["o"], "config2 B4H32N4096", "O")
    parity.check_torch(dq, refs["dq"], "config2 B4H32N4096", "dQ")
    parity.check_torch(dk, refs["dk"], "config2 B4H32N4096", "dK")
    parity.check_torch(dv, refs["dv"], "config2 B4H32N4096", "dV")


def test_headline_32k_sampled_heads(cuda_device):
    """The metric's configuration B1 H32 N32768 (all heads run), heads 0 and 21 checked
    against the reference's dense branch (N < 2**16)."""
    import torch
    B, H, N = 1, 32, 32768
    q, k, v, do = _inputs(cuda_device, 32, B, H, N, q_scale=D ** -0.5)
    ours = _ours(q, k, v, do)
    for h in (0, 21):
        hs = slice(h, h + 1)
        r = _reference(q, k, v, do, 0, hs)
        _compare(f"32K B1H32 head {h}", ours, r, 0, hs)
        del r
        torch.cuda.empty_cache()


def test_blockwise_branch_65536(cuda_device):
    """N = 2**16, one head: the reference's blockwise Lucid_Tril_Solver branch."""
    from oracle import torch_blockwise as tb
    assert tb.reference_block_size(65536) == 2 ** 14
    q, k, v, do = _inputs(cuda_device, 64, 1, 1, 65536, q_scale=D ** -0.5)
    ours = _ours(q, k, v, do)
    r = _reference(q, k, v, do, 0, slice(0, 1))
    _compare("N65536 blockwise", ours, r, 0, slice(0, 1))


def test_stress_128k_correlated_keys(cuda_device):
    """N = 131072, one head, K = 0.6 s + 0.8 n: the solved values X, O and the gradients
    against the blockwise float32 reference."""
    import torch
    from lucid_b200 import solve_fwd
    N = 131072
    q, k, v, do = _inputs(cuda_device, 128, 1, 1, N, keys="corr")
    x = solve_fwd(k, v, D ** -0.5, 1e-5)[0]
    torch.cuda.synchronize()
    ours = _ours(q, k, v, do)
    r = _reference(q, k, v, do, 0, slice(0, 1))
    parity.check_torch(x[0, :, :N], r["x"], "128K stress", "X")
    _compare("128K stress", ours, r, 0, slice(0, 1))


def test_path_16384_one_head(cuda_device):
    """LUCID-Path at the config-3 sequence length T = 16384 (one batch, one head, q = k)
    against the float64 block restatement: o, dk, dv within the strict bar, every
    gradient within 2 % of its largest magnitude."""
    import torch
    from lucid_b200.path import parallel_lucid_path_attention
    from oracle.path_oracle import make_path_inputs, path_bwd_blockwise, path_fwd_blockwise
    d = make_path_inputs(16384, 1, 16384, 1, 128)
    o_ref, _ = path_fwd_blockwise(d["k"], d["v"], d["w"], d["beta"])
    _, dk_ref, dv_ref, dw_ref, db_ref = path_bwd_blockwise(d["k"], d["v"], d["w"], d["beta"], d["do"])
    t = {n: torch.tensor(d[n], dtype=torch.float32).to(cuda_device, torch.bfloat16).requires_grad_(True)
         for n in ("k", "v", "w", "beta")}
    o, _ = parallel_lucid_path_attention(t["k"], t["v"], t["w"], t["beta"])
    o.backward(torch.tensor(d["do"], dtype=torch.float32).to(cuda_device, torch.bfloat16))
    torch.cuda.synchronize()
    f = lambda a: a.detach().float().cpu().numpy()
    parity.check(f(o), o_ref, "path T16384", "o")
    for name, key, ref in (("dk", "k", dk_ref), ("dv", "v", dv_ref), ("dw", "w", dw_ref), ("dbeta", "beta", db_ref)):
        g = f(t[key].grad)
        parity.check(g, ref, "path T16384", name)
        rel = np.abs(g - ref).max() / max(np.abs(ref).max(), 1e-30)
        assert rel <= 2e-2, f"path T16384 {name}: rel {rel:.3e}"
