"""GPU parity tests: the sm_100a kernels (through the C ABI) against the CPU
oracle and the reference's golden fixtures.

Tolerance (bf16, tests/parity.py): max |ours - ref| <= 1e-2 + ulp_bf16(ref)/2,
i.e. the op's max-abs 1e-2 before the final rounding of the bf16 output (no bf16
value is closer to ref than half an ulp), and the earlier 1e-2 + 2^-8 |ref| as a
second check; the reference value is the float64 restatement of
modeling_lucid.py on the same (bf16-exact) inputs.  For grouped-query heads the
kv-head gradients dK and dV are sums over the G query heads of a group, each
carrying the bf16 rounding of the attention probabilities, so their absolute
budget is 1e-2 * sqrt(G).
"""
import numpy as np
import pytest

import parity
from conftest import ATTN_CASES, load_golden
from oracle import lucid_oracle as orc

pytestmark = pytest.mark.gpu


def _t(a, dev, dtype=None):
    import torch
    return torch.as_tensor(np.ascontiguousarray(a)).to(device=dev, dtype=dtype or torch.bfloat16)


def _np(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def assert_bf16_close(ours, ref, what, group=1):
    return parity.check(ours, ref, "small", what, group)


def _rand_inputs(seed, B, Hq, Hkv, N, D=128, keys="iid", q_scale=1.0):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, Hq, N, D)) * q_scale
    if keys == "iid":
        k = rng.standard_normal((B, Hkv, N, D))
    else:
        k = 0.6 * rng.standard_normal((B, Hkv, 1, D)) + 0.8 * rng.standard_normal((B, Hkv, N, D))
    v = rng.standard_normal((B, Hkv, N, D))
    do = rng.standard_normal((B, N, Hq, D))
    import torch
    rnd = lambda a: torch.as_tensor(a).to(torch.bfloat16).double().numpy()
    return [rnd(a) for a in (q, k, v, do)]


# ---------------------------------------------------------------------------
# tensor-core primitive
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("via_tma", [0, 1, 2])
@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_umma_tile_selftest(cuda_device, a_mn, b_mn, via_tma):
    if via_tma == 2 and a_mn:
        pytest.skip("A from TMEM is always K-major")
    import torch
    from lucid_b200 import _lib
    lib = _lib.load()
    g = torch.Generator(device="cpu").manual_seed(0)
    a = torch.randn(128, 128, generator=g).to(torch.bfloat16)
    b = torch.randn(128, 128, generator=g).to(torch.bfloat16)
    da, db = a.to(cuda_device), b.to(cuda_device)
    d = torch.zeros(128 * 128 + 4, dtype=torch.float32, device=cuda_device)
    rc = lib.lucid_selftest_umma(da.data_ptr(), db.data_ptr(), d.data_ptr(), a_mn, b_mn, via_tma,
                                 torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    af, bf = a.float(), b.float()
    A = af.t() if a_mn else af
    Bm = bf if b_mn else bf.t()
    ref = A @ Bm
    got = d[: 128 * 128].view(128, 128).cpu()
    assert d[128 * 128:].view(torch.int32)[0].item() == 0
    torch.testing.assert_close(got, ref, atol=1e-3, rtol=1e-3)


# ---------------------------------------------------------------------------
# solve forward
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("B,H,N,keys", [(1, 1, 128, "iid"), (1, 2, 130, "iid"), (2, 3, 512, "iid"),
                                        (1, 2, 1000, "corr"), (1, 1, 2048, "iid")])
def test_solve_fwd_matches_oracle(cuda_device, B, H, N, keys):
    from lucid_b200 import solve_fwd
    _, k, v, _ = _rand_inputs(10 + N, B, H, H, N, keys=keys)
    s = 128 ** -0.5
    x, khat, u, rstd, dinv = solve_fwd(_t(k, cuda_device), _t(v, cuda_device), s, 1e-5)
    ref = orc.solve(k, v, s, 1e-5)
    kh, r = orc.rms_norm(k, 1e-5)
    np.testing.assert_allclose(_np(rstd)[..., :N], r[..., 0], rtol=1e-5)
    assert_bf16_close(_np(khat)[:, :, :N], kh, "khat")
    assert_bf16_close(_np(x)[:, :, :N], ref, "X")
    assert np.all(np.isfinite(_np(x)))


@pytest.mark.parametrize("B,H,N,keys", [(1, 1, 1, "iid"), (1, 1, 128, "iid"), (1, 2, 257, "corr"),
                                        (2, 3, 1000, "iid"), (1, 2, 4096, "corr")])
def test_solve_fwd_chain_and_wavefront_schedules(cuda_device, monkeypatch, B, H, N, keys):
    """Both schedules of the solve forward against the oracle, and against each other
    (the chain schedule only regroups the fp32 row sums)."""
    from lucid_b200 import _lib, solve_fwd
    lib = _lib.load()
    _, k, v, _ = _rand_inputs(20 + N, B, H, H, N, keys=keys)
    s = 128 ** -0.5
    ref = orc.solve(k, v, s, 1e-5)
    xs = {}
    for sched in ("chain", "wavefront"):
        monkeypatch.setenv("LUCID_B200_SOLVE_SCHEDULE", sched)
        base = lib.lucid_solve_fwd_workspace_bytes(B, H, N, 128)
        fast = lib.lucid_solve_fwd_fast_workspace_bytes(B, H, N, 128)
        assert (fast > base) == (sched == "chain")
        x = solve_fwd(_t(k, cuda_device), _t(v, cuda_device), s, 1e-5)[0]
        _lib.check_status()
        xs[sched] = _np(x)[:, :, :N]
        assert np.all(np.isfinite(xs[sched]))
        assert_bf16_close(xs[sched], ref, f"X ({sched})")
    diff = np.abs(xs["chain"] - xs["wavefront"])
    assert float(diff.max()) <= 2e-2 * max(1.0, float(np.abs(ref).max()))


@pytest.mark.parametrize("sched", ["chain", "wavefront"])
@pytest.mark.parametrize("B,Hq,Hkv,N", [(1, 2, 2, 1000), (2, 4, 2, 300), (1, 8, 2, 2048), (1, 1, 1, 128)])
def test_fused_fwd_equals_two_stages(cuda_device, monkeypatch, sched, B, Hq, Hkv, N):
    """lucid_fused_fwd (one launch under the chain schedule, two under the wavefront) gives
    exactly the solve's and the attention's outputs of the separate calls."""
    import torch
    from lucid_b200 import _lib, attn_fwd, fused_fwd, solve_fwd
    monkeypatch.setenv("LUCID_B200_SOLVE_SCHEDULE", sched)
    q, k, v, _ = _rand_inputs(30 + N, B, Hq, Hkv, N, q_scale=128 ** -0.5)
    qd, kd, vd = _t(q, cuda_device), _t(k, cuda_device), _t(v, cuda_device)
    s = 128 ** -0.5
    x1, kh1, u1, r1, d1 = solve_fwd(kd, vd, s, 1e-5)
    o1, lse1, res1 = attn_fwd(qd, kd, x1, s, residual=True)
    x2, kh2, u2, r2, d2, o2, lse2, res2 = fused_fwd(qd, kd, vd, s, 1e-5)
    _lib.check_status()
    Np = x1.shape[2]
    # rows from N on are padding, not written
    for name, a, b_ in (("x", x1, x2), ("khat", kh1, kh2), ("u", u1, u2), ("rstd", r1, r2), ("dinv", d1, d2),
                        ("lse", lse1, lse2)):
        assert torch.equal(a[:, :, :N], b_[:, :, :N]), name
    assert torch.equal(o1, o2) and torch.equal(res1, res2)
    assert Np == x2.shape[2]
    ref = orc.lucid_fwd(q, k, v, s, 1e-5)[0]
    assert_bf16_close(_np(o2), ref, f"O (fused, {sched})")


def test_solve_fwd_diag_block_inverse(cuda_device):
    """U = (I + L~)^-1 - I of every diagonal block, against numpy."""
    from lucid_b200 import solve_fwd
    _, k, v, _ = _rand_inputs(3, 1, 1, 1, 256, keys="corr")
    s = 128 ** -0.5
    _, _, u, _, dinv = solve_fwd(_t(k, cuda_device), _t(v, cuda_device), s, 1e-5)
    p = orc.build_p(k, s, 1e-5)[0, 0]
    un = _np(u)[0, 0]
    for i in range(2):
        blk = p[i * 128:(i + 1) * 128, i * 128:(i + 1) * 128]
        d = np.diag(blk)
        lt = np.tril(blk, -1) / d[:, None]
        want = np.linalg.inv(np.eye(128) + lt) - np.eye(128)
        np.testing.assert_allclose(un[i * 128:(i + 1) * 128], want, atol=2e-3)
        np.testing.assert_allclose(_np(dinv)[0, 0, i * 128:(i + 1) * 128], 1.0 / d, rtol=1e-5)


# ---------------------------------------------------------------------------
# full op against the reference's own outputs
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("case", ATTN_CASES)
def test_fused_matches_reference_fixture(cuda_device, case):
    """Every reference fixture, head_dim 128 and the zero-padded head_dim 32."""
    import torch
    from lucid_b200 import lucid_attention
    g = load_golden(case)
    q = _t(g["q"], cuda_device).requires_grad_(True)
    k = _t(g["k"], cuda_device).requires_grad_(True)
    v = _t(g["v"], cuda_device).requires_grad_(True)
    o = lucid_attention(q, k, v, float(g["scale"]), float(g["eps"]))
    o.backward(_t(g["do"], cuda_device))
    torch.cuda.synchronize()
    G = g["q"].shape[1] // g["k"].shape[1]
    assert_bf16_close(_np(o), g["o"], f"{case} O")
    assert_bf16_close(_np(q.grad), g["dq"], f"{case} dQ")
    assert_bf16_close(_np(k.grad), g["dk"], f"{case} dK", G)
    assert_bf16_close(_np(v.grad), g["dv"], f"{case} dV", G)


@pytest.mark.parametrize("B,Hq,Hkv,N,keys,qs,D", [
    (1, 2, 2, 384, "iid", 1.0, 128),
    (2, 4, 2, 300, "iid", 128 ** -0.5, 128),
    (1, 1, 1, 1024, "corr", 1.0, 128),
    (1, 8, 1, 256, "iid", 1.0, 128),
    (1, 8, 1, 640, "corr", 1.0, 68),    # the reference model's head_dim (lucid/config), 8 q per kv head
    (2, 2, 2, 200, "iid", 1.0, 64),
])
def test_fused_fwd_bwd_matches_oracle(cuda_device, B, Hq, Hkv, N, keys, qs, D):
    """Head dimensions below 128 run zero-padded: the oracle normalises K over
    the true D and uses s = D^-1/2."""
    import torch
    from lucid_b200 import lucid_attention
    q_, k_, v_, do_ = _rand_inputs(100 + N, B, Hq, Hkv, N, D=D, keys=keys, q_scale=qs)
    s = D ** -0.5
    q = _t(q_, cuda_device).requires_grad_(True)
    k = _t(k_, cuda_device).requires_grad_(True)
    v = _t(v_, cuda_device).requires_grad_(True)
    o = lucid_attention(q, k, v, s)
    o.backward(_t(do_, cuda_device))
    torch.cuda.synchronize()
    o_ref, dq_ref, dk_ref, dv_ref = orc.lucid_fwd_bwd(q_, k_, v_, do_, s)
    G = Hq // Hkv
    assert_bf16_close(_np(o), o_ref, "O")
    assert_bf16_close(_np(q.grad), dq_ref, "dQ")
    assert_bf16_close(_np(k.grad), dk_ref, "dK", G)
    assert_bf16_close(_np(v.grad), dv_ref, "dV", G)


@pytest.mark.parametrize("B,Hq,Hkv,N", [(1, 2, 2, 1000), (2, 4, 1, 384)])
def test_attn_bwd_stored_tiles_equal_recompute(cuda_device, monkeypatch, B, Hq, Hkv, N):
    """The stored-tile schedule streams the column pass's own bf16 dS^T tiles through
    the row pass in the recomputing pass's key-block order: bit-identical results."""
    import torch
    from lucid_b200 import attn_bwd, attn_fwd, solve_fwd
    q_, k_, v_, do_ = _rand_inputs(31 + N, B, Hq, Hkv, N)
    q, k, v, do = (_t(a, cuda_device) for a in (q_, k_, v_, do_))
    s = 128 ** -0.5
    x = solve_fwd(k, v, s, 1e-5)[0]
    o, lse = attn_fwd(q, k, x, s)
    out = {}
    for mode in ("0", "1"):
        monkeypatch.setenv("LUCID_B200_STORED_TILES", mode)
        out[mode] = attn_bwd(q, k, x, o, do, lse, s)
        torch.cuda.synchronize()
    for a, b in zip(out["0"], out["1"]):
        assert torch.equal(a, b)


@pytest.mark.parametrize("B,H,N,keys", [(1, 2, 1000, "corr"), (2, 1, 384, "iid"), (1, 1, 128, "iid")])
def test_solve_bwd_stored_tiles_equal_recompute(cuda_device, monkeypatch, B, H, N, keys):
    """Solve backward: the stored dG^T tiles streamed through the row pass give the
    recomputing schedule's results bit for bit (N = 128: a single block, no tiles)."""
    import torch
    from lucid_b200 import solve_bwd, solve_fwd
    _, k_, v_, _ = _rand_inputs(47 + N, B, H, H, N, keys=keys)
    k, v = _t(k_, cuda_device), _t(v_, cuda_device)
    s = 128 ** -0.5
    x, khat, u, rstd, dinv = solve_fwd(k, v, s, 1e-5)
    g = torch.Generator(device="cpu").manual_seed(N)
    dx = torch.randn(x.shape, generator=g).to(cuda_device)
    out = {}
    for mode in ("0", "1"):
        monkeypatch.setenv("LUCID_B200_STORED_TILES", mode)
        out[mode] = solve_bwd(k, x, khat, u, rstd, dinv, dx, s)
        torch.cuda.synchronize()
    for a, b in zip(out["0"], out["1"]):
        assert torch.equal(a, b)


def test_separate_functions_compose(cuda_device):
    """get_v_prime (LucidSolveFunction) followed by the attention function
    (LucidAttnFunction) gives the same result as the fused op."""
    import torch
    from lucid_b200 import LucidAttnFunction, LucidSolveFunction
    q_, k_, v_, do_ = _rand_inputs(7, 1, 2, 2, 200)
    s = 128 ** -0.5
    q = _t(q_, cuda_device).requires_grad_(True)
    k = _t(k_, cuda_device).requires_grad_(True)
    v = _t(v_, cuda_device).requires_grad_(True)
    x = LucidSolveFunction.apply(k, v, s, 1e-5)
    o = LucidAttnFunction.apply(q, k, x, s)
    o.backward(_t(do_, cuda_device))
    torch.cuda.synchronize()
    o_ref, dq_ref, dk_ref, dv_ref = orc.lucid_fwd_bwd(q_, k_, v_, do_, s)
    assert_bf16_close(_np(o), o_ref, "O")
    assert_bf16_close(_np(q.grad), dq_ref, "dQ")
    # dX crosses the autograd boundary in bf16 here: allow one more rounding
    assert_bf16_close(_np(k.grad), dk_ref, "dK")
    assert_bf16_close(_np(v.grad), dv_ref, "dV")


def test_forward_is_deterministic(cuda_device):
    import torch
    from lucid_b200 import lucid_attention
    q_, k_, v_, _ = _rand_inputs(5, 1, 4, 4, 640)
    q, k, v = (_t(a, cuda_device) for a in (q_, k_, v_))
    o1 = lucid_attention(q, k, v)
    o2 = lucid_attention(q, k, v)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)


def test_strided_bnhd_inputs(cuda_device):
    """Q/K/V as transposed views of [B, N, H, D] projections (the layout
    LucidAttention.forward produces, modeling_lucid.py:433-435)."""
    import torch
    from lucid_b200 import lucid_attention
    q_, k_, v_, do_ = _rand_inputs(9, 2, 2, 2, 256)
    mk = lambda a: _t(np.ascontiguousarray(np.swapaxes(a, 1, 2)), cuda_device).transpose(1, 2)
    q, k, v = mk(q_), mk(k_), mk(v_)
    assert not q.is_contiguous()
    o = lucid_attention(q, k, v)
    torch.cuda.synchronize()
    o_ref, _ = orc.lucid_fwd(q_, k_, v_, 128 ** -0.5)
    assert_bf16_close(_np(o), o_ref, "O")


# ---------------------------------------------------------------------------
# stage-level checks (each backward pass against the oracle in isolation)
# ---------------------------------------------------------------------------
def _attn_bwd_oracle(q, k, x, do, s):
    """dQ, dK, dX of sum(O * dO), O = softmax(s Q K^T + causal) X (float64)."""
    B, Hq, N, D = q.shape
    Hkv = k.shape[1]
    g = Hq // Hkv
    kr, xr = np.repeat(k, g, axis=1), np.repeat(x, g, axis=1)
    sc = np.einsum("bhld,bhsd->bhls", q, kr) * s
    sc = np.where(np.tril(np.ones((N, N), dtype=bool)), sc, -np.inf)
    a = np.exp(sc - sc.max(-1, keepdims=True))
    a /= a.sum(-1, keepdims=True)
    dot = np.swapaxes(do, 1, 2)
    da = dot @ np.swapaxes(xr, -1, -2)
    ds = a * (da - np.sum(da * a, -1, keepdims=True))
    dq = s * ds @ kr
    dk = (s * np.swapaxes(ds, -1, -2) @ q).reshape(B, Hkv, g, N, D).sum(2)
    dx = (np.swapaxes(a, -1, -2) @ dot).reshape(B, Hkv, g, N, D).sum(2)
    return dq, dk, dx


@pytest.mark.parametrize("B,Hq,Hkv,N,keys", [(1, 1, 1, 256, "corr"), (1, 2, 1, 384, "iid"),
                                             (1, 2, 2, 300, "corr")])
def test_attn_bwd_stage(cuda_device, B, Hq, Hkv, N, keys):
    import torch
    from lucid_b200 import attn_bwd, attn_fwd, padded_len
    q_, k_, v_, do_ = _rand_inputs(300 + N, B, Hq, Hkv, N, keys=keys)
    s = 128 ** -0.5
    x_ = torch.as_tensor(orc.solve(k_, v_, s, 1e-5)).to(torch.bfloat16).double().numpy()
    xp = np.zeros((B, Hkv, padded_len(N), 128))
    xp[:, :, :N] = x_
    q, k, do = _t(q_, cuda_device), _t(k_, cuda_device), _t(do_, cuda_device)
    x = _t(xp, cuda_device)
    o, lse, o_res = attn_fwd(q, k, x, s, residual=True)
    dq, dk, dx = attn_bwd(q, k, x, o, do, lse, s, o_res=o_res)
    torch.cuda.synchronize()
    dq_r, dk_r, dx_r = _attn_bwd_oracle(q_, k_, x_, do_, s)
    G = Hq // Hkv
    assert_bf16_close(_np(dq), dq_r, "dQ")
    assert_bf16_close(_np(dk)[:, :, :N], dk_r, "dK(attn)", G)
    assert_bf16_close(_np(dx)[:, :, :N], dx_r, "dX", G)


@pytest.mark.parametrize("B,H,N,keys", [(1, 1, 256, "corr"), (1, 2, 384, "corr"), (2, 1, 200, "iid")])
def test_solve_bwd_stage(cuda_device, B, H, N, keys):
    """dV = P^-T dX and dK through P and RMSNorm, given dX (fp32)."""
    import torch
    from lucid_b200 import padded_len, solve_bwd, solve_fwd
    _, k_, v_, _ = _rand_inputs(400 + N, B, H, H, N, keys=keys)
    s = 128 ** -0.5
    rng = np.random.default_rng(N)
    dx_ = rng.standard_normal((B, H, N, 128))
    k, v = _t(k_, cuda_device), _t(v_, cuda_device)
    x, khat, u, rstd, dinv = solve_fwd(k, v, s, 1e-5)
    dxp = torch.zeros(B, H, padded_len(N), 128, dtype=torch.float32, device=cuda_device)
    dxp[:, :, :N] = torch.as_tensor(dx_, dtype=torch.float32, device=cuda_device)
    dk, dv = solve_bwd(k, x, khat, u, rstd, dinv, dxp, s)
    torch.cuda.synchronize()
    p = orc.build_p(k_, s, 1e-5)
    xo = orc.solve(k_, v_, s, 1e-5)
    dv_r = np.linalg.solve(np.swapaxes(p, -1, -2), dx_)
    kh, r = orc.rms_norm(k_, 1e-5)
    dg = s * p * (-np.tril(dv_r @ np.swapaxes(xo, -1, -2)))
    dkh = dg @ kh + np.swapaxes(dg, -1, -2) @ kh
    dk_r = r * (dkh - np.sum(kh * dkh, -1, keepdims=True) / 128 * kh)
    assert_bf16_close(_np(dv), dv_r, "dV")
    assert_bf16_close(_np(dk), dk_r, "dK(solve)")
