"""LUCID-Path on the B200 kernels against the reference and the oracle.

Reference: the fixtures of tests/golden/make_path_golden.py (the reference's
Triton op in float32).  Oracle: oracle/path_oracle.py (float64).  The kernels
compute in bf16 with fp32 accumulation, so the bars are:

  o:          max |o - ref| <= 1e-2 (the op's bf16 tolerance) + 2^-8 |ref|, or,
              where the path scores are large (scale 0.15), no more than 1.5x
              the deviation of the reference's own bf16 forward, modelled by
              oracle/path_precision.py
  gradients:  max |g - ref| <= 2e-2 * max |ref|   (the gradients of the
              default-scale fixtures are ~1e-3 in magnitude, so an absolute
              1e-2 bar would be vacuous; the bar is relative to their scale)
"""
import numpy as np
import pytest

from conftest import PATH_ATTN_CASES, PATH_CASES, load_path_golden

pytestmark = pytest.mark.gpu

GRADS = ("dq", "dk", "dv", "dw", "dbeta")


def _to(torch, a, dev, dtype=None):
    return torch.tensor(a, dtype=torch.float32).to(dev, dtype or torch.bfloat16)


def _run(torch, d, dev, scale=None, backward=True):
    from lucid_b200.path import parallel_lucid_path_attention
    k = _to(torch, d["k"], dev).requires_grad_(backward)
    v = _to(torch, d["v"], dev).requires_grad_(backward)
    w = _to(torch, d["w"], dev).requires_grad_(backward)
    beta = _to(torch, d["beta"], dev).requires_grad_(backward)
    q = _to(torch, d["q"], dev).requires_grad_(backward) if d.get("q") is not None else None
    o, kc = parallel_lucid_path_attention(k, v, w, beta, q=q, scale=scale)
    assert kc is None
    out = {"o": o.detach().float().cpu().numpy()}
    if backward:
        o.backward(_to(torch, d["do"], dev))
        torch.cuda.synchronize()
        out.update(dk=k.grad.float().cpu().numpy(), dv=v.grad.float().cpu().numpy(),
                   dw=w.grad.float().cpu().numpy(), dbeta=beta.grad.float().cpu().numpy())
        if q is not None:
            out["dq"] = q.grad.float().cpu().numpy()
    return out


def _check(got, ref, label, ref_dev=None):
    o, ro = got["o"], ref["o"]
    assert np.all(np.isfinite(o)), label
    if ref_dev is None:
        err = np.abs(o - ro) - (1e-2 + 2.0 ** -8 * np.abs(ro))
        assert err.max() <= 0, f"{label} o: max err {np.abs(o - ro).max():.3e}"
    else:
        dev = np.abs(o - ro).max()
        assert dev <= max(1.5 * ref_dev, 1e-2), f"{label} o: max err {dev:.3e}, reference model {ref_dev:.3e}"
    for nm in GRADS:
        if nm not in ref or nm not in got:
            continue
        g, r = got[nm], ref[nm]
        assert np.all(np.isfinite(g)), f"{label} {nm}"
        rel = np.abs(g - r).max() / max(np.abs(r).max(), 1e-30)
        assert rel <= 2e-2, f"{label} {nm}: max err {np.abs(g - r).max():.3e} (rel {rel:.3e})"


@pytest.mark.parametrize("name", PATH_CASES)
def test_path_matches_reference_fixture(cuda_device, name):
    torch = pytest.importorskip("torch")
    d = load_path_golden(name)
    got = _run(torch, d, cuda_device)
    _check(got, d, name)


@pytest.mark.parametrize("B,T,H,HQ,with_q,scale", [
    (1, 300, 1, 1, False, 0.15),     # ragged T, large path scores
    (2, 256, 2, 2, False, 0.15),     # two batches, two heads
    (1, 260, 1, 2, True, 0.15),      # grouped query heads with explicit q
    (1, 128, 1, 1, False, 0.15),     # a single block (diagonal only)
    (1, 77, 2, 2, False, None),      # shorter than one block, default scale
])
def test_path_matches_oracle(cuda_device, B, T, H, HQ, with_q, scale):
    torch = pytest.importorskip("torch")
    from oracle.path_oracle import make_path_inputs, path_fwd_bwd_torch
    d = make_path_inputs(100 + T + HQ, B, T, H, 128, HQ, with_q)
    o, dq, dk, dv, dw, db = path_fwd_bwd_torch(d["k"], d["v"], d["w"], d["beta"], d["do"], q=d["q"], scale=scale)
    ref = dict(o=o, dk=dk, dv=dv, dw=dw, dbeta=db)
    if dq is not None:
        ref["dq"] = dq
    got = _run(torch, d, cuda_device, scale=scale)
    ref_dev = None
    if scale is not None:
        from oracle.path_precision import reference_bf16_forward
        om = reference_bf16_forward(d["k"], d["v"], d["w"], d["beta"], q=d["q"], scale=scale)
        ref_dev = float(np.abs(om - o).max())
    _check(got, ref, f"B{B} T{T} H{H} HQ{HQ}", ref_dev)


def test_path_forward_long_sequence_matches_oracle(cuda_device):
    """16 row blocks: the wavefront solve and the score chain over many blocks."""
    torch = pytest.importorskip("torch")
    from oracle.path_oracle import make_path_inputs, path_fwd
    d = make_path_inputs(5, 1, 2048, 1, 128)
    from oracle.path_precision import reference_bf16_forward
    ref, _ = path_fwd(d["k"], d["v"], d["w"], d["beta"], scale=0.15)
    ref_dev = float(np.abs(reference_bf16_forward(d["k"], d["v"], d["w"], d["beta"], scale=0.15) - ref).max())
    got = _run(torch, d, cuda_device, scale=0.15, backward=False)
    _check(got, {"o": ref}, "T2048", ref_dev)


def test_path_solve_is_linear_in_v(cuda_device):
    """O = (I + L)^-1 V is linear in V at the benchmark's block count."""
    torch = pytest.importorskip("torch")
    from lucid_b200.path import parallel_lucid_path_attention
    g = torch.Generator(device="cpu").manual_seed(3)
    B, T, H = 1, 4096, 2
    k = torch.randn(B, T, H, 128, generator=g)
    w = torch.nn.functional.normalize(torch.randn(B, T, H, 128, generator=g), dim=-1)
    beta = 2 * torch.sigmoid(torch.randn(B, T, H, generator=g))
    v1 = torch.randn(B, T, H, 128, generator=g)
    v2 = torch.randn(B, T, H, 128, generator=g)
    dev = cuda_device
    k, w, beta = (t.to(dev, torch.bfloat16) for t in (k, w, beta))
    with torch.no_grad():
        o1, _ = parallel_lucid_path_attention(k, v1.to(dev, torch.bfloat16), w, beta, scale=0.15)
        o2, _ = parallel_lucid_path_attention(k, v2.to(dev, torch.bfloat16), w, beta, scale=0.15)
        o12, _ = parallel_lucid_path_attention(k, (v1 + v2).to(dev, torch.bfloat16), w, beta, scale=0.15)
    # bf16 outputs and operands: linear up to a few bf16 ulps of |o|
    diff = (o12.float() - o1.float() - o2.float()).abs().max().item()
    assert diff < 1e-2 * o12.float().abs().max().item(), diff
    assert torch.isfinite(o12).all()


def test_path_deterministic(cuda_device):
    torch = pytest.importorskip("torch")
    from oracle.path_oracle import make_path_inputs
    d = make_path_inputs(9, 1, 384, 1, 128)
    a = _run(torch, d, cuda_device, scale=0.15)
    b = _run(torch, d, cuda_device, scale=0.15)
    for nm in ("o", "dk", "dv", "dw", "dbeta"):
        np.testing.assert_array_equal(a[nm], b[nm])


def test_path_varlen_matches_separate_sequences(cuda_device):
    """cu_seqlens: sequences of 150, 250, 100, 300 and 10 tokens (block counts 2, 2, 1, 3
    and 1, so three batched groups) against one call per sequence: o, the key cache and
    every gradient."""
    torch = pytest.importorskip("torch")
    from lucid_b200.path import parallel_lucid_path_attention
    from oracle.path_oracle import make_path_inputs
    bounds = [0, 150, 400, 500, 800, 810]
    d = make_path_inputs(21, 1, bounds[-1], 2, 128)
    dev = cuda_device
    base = [_to(torch, d[n], dev) for n in ("k", "v", "w", "beta")]
    do = _to(torch, d["do"], dev)

    def run(sl):
        leaves = [t[:, sl].clone().requires_grad_(True) for t in base]
        return leaves

    cu = torch.tensor(bounds, dtype=torch.int32, device=dev)
    packed = run(slice(None))
    o, kc = parallel_lucid_path_attention(*packed, cu_seqlens=cu, scale=0.15, use_cache=True)
    o.backward(do)
    for a, b in zip(bounds[:-1], bounds[1:]):
        sep = run(slice(a, b))
        o_s, kc_s = parallel_lucid_path_attention(*sep, scale=0.15, use_cache=True)
        o_s.backward(do[:, a:b])
        torch.testing.assert_close(o[:, a:b], o_s, rtol=0, atol=0)
        torch.testing.assert_close(kc[:, a:b], kc_s, rtol=0, atol=0)
        for t_p, t_s in zip(packed, sep):
            torch.testing.assert_close(t_p.grad[:, a:b], t_s.grad, rtol=0, atol=0)


def _attn(torch, d, dev, scale=None):
    from lucid_b200.path import parallel_path_attention_fwd
    k, v, w, beta = (_to(torch, d[n], dev) for n in ("k", "v", "w", "beta"))
    q = _to(torch, d["q"], dev) if d.get("q") is not None else None
    o, lse = parallel_path_attention_fwd(q, k, v, w, beta, scale=scale)
    torch.cuda.synchronize()
    return o.float().cpu().numpy(), lse.cpu().numpy()


@pytest.mark.parametrize("name", PATH_ATTN_CASES)
def test_path_attention_matches_reference_fixture(cuda_device, name):
    torch = pytest.importorskip("torch")
    d = load_path_golden(name)
    o, lse = _attn(torch, d, cuda_device)
    assert np.all(np.isfinite(o)) and np.all(np.isfinite(lse))
    err = np.abs(o - d["o"]) - (1e-2 + 2.0 ** -8 * np.abs(d["o"]))
    assert err.max() <= 0, np.abs(o - d["o"]).max()
    assert np.abs(lse - d["lse"]).max() < 2e-2


@pytest.mark.parametrize("B,T,H,HQ,with_q,scale", [(1, 1000, 1, 1, False, None), (2, 300, 2, 4, True, 0.2),
                                                     (1, 64, 1, 1, False, None)])
def test_path_attention_matches_oracle(cuda_device, B, T, H, HQ, with_q, scale):
    """Many blocks (T = 1000: 8 blocks, rescaling of the running maximum), GQA with an
    explicit q and sharper scores, a sequence shorter than one block.  Bar: 1e-2, or
    1.5x the deviation of the reference's own bf16 kernels (oracle/path_precision.py)
    where that is larger."""
    torch = pytest.importorskip("torch")
    from oracle.path_oracle import make_path_inputs, path_attention_fwd
    from oracle.path_precision import reference_bf16_attention
    d = make_path_inputs(40 + T, B, T, H, 128, HQ, with_q)
    ro, rl = path_attention_fwd(d["k"], d["v"], d["w"], d["beta"], q=d["q"], scale=scale)
    ref_dev = float(np.abs(reference_bf16_attention(d["k"], d["v"], d["w"], d["beta"], q=d["q"],
                                                    scale=scale) - ro).max())
    o, lse = _attn(torch, d, cuda_device, scale=scale)
    dev = float(np.abs(o - ro).max())
    assert np.all(np.isfinite(o))
    assert dev <= max(1.5 * ref_dev, 1e-2), (dev, ref_dev)
    assert np.abs(lse - rl).max() < 2e-2


def test_path_head_groups_match_whole_batch(cuda_device, monkeypatch):
    """The bounded-memory schedule (kv-head groups one after another, the backward
    recomputing each group's forward) against the whole-batch call: o, the key cache
    and every gradient bit-identical (B2, 2 kv heads, 4 query heads, explicit q)."""
    torch = pytest.importorskip("torch")
    from lucid_b200 import _lib
    from lucid_b200.path import parallel_lucid_path_attention, path_memory_groups
    from oracle.path_oracle import make_path_inputs
    d = make_path_inputs(33, 2, 300, 2, 128, 4, True)
    dev = cuda_device
    base = [_to(torch, d[n], dev) for n in ("q", "k", "v", "w", "beta")]
    do = _to(torch, d["do"], dev)

    def run():
        leaves = [t.clone().requires_grad_(True) for t in base]
        o, kc = parallel_lucid_path_attention(leaves[1], leaves[2], leaves[3], leaves[4], q=leaves[0],
                                              use_cache=True)
        o.backward(do)
        torch.cuda.synchronize()
        return [o, kc] + [t.grad for t in leaves]

    whole = run()
    lib = _lib.load()
    one_head = lib.lucid_path_fwd_workspace_bytes(1, 300, 1, 2, 128) + lib.lucid_path_bwd_workspace_bytes(1, 300, 1, 2, 128)
    monkeypatch.setenv("LUCID_B200_PATH_MAX_BYTES", str(one_head))
    assert len(path_memory_groups(2, 300, 2, 4, dev)) == 4
    grouped = run()
    for a, b in zip(whole, grouped):
        torch.testing.assert_close(a, b, rtol=0, atol=0)
