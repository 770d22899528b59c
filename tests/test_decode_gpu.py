"""Decoding on the B200 kernels: get_new_v_prime (modeling_lucid.py:576-598)
against the reference's own outputs, decode attention against the oracle, the
LucidAttention mirror stepping through a cache, and the LUCID-Path decode-time
key cache (prepare_k_cache.py) against the reference's Triton op."""
import numpy as np
import pytest

from conftest import DECODE_CASES, PATH_CASES, load_decode_golden, load_path_golden

pytestmark = pytest.mark.gpu


def _bf(torch, a, dev):
    return torch.tensor(a, dtype=torch.float32).to(dev, torch.bfloat16)


@pytest.mark.parametrize("name", DECODE_CASES)
def test_decode_update_matches_reference_fixture(cuda_device, name):
    torch = pytest.importorskip("torch")
    from lucid_b200 import decode_update
    d = load_decode_golden(name)
    t = {n: _bf(torch, d[n], cuda_device) for n in ("k_new", "v_new", "k_cache", "x_cache")}
    x = decode_update(t["k_new"], t["v_new"], t["k_cache"], t["x_cache"], float(d["scale"]), float(d["eps"]))
    x = x.float().cpu().numpy()
    err = np.abs(x - d["x_new"]) - (1e-2 + 2.0 ** -8 * np.abs(d["x_new"]))
    assert err.max() <= 0, np.abs(x - d["x_new"]).max()


@pytest.mark.parametrize("B,H,Ln,Nc,D", [(1, 4, 1, 3000, 68), (2, 2, 3, 500, 68), (1, 2, 2, 700, 32)])
def test_decode_update_small_head_dim_matches_oracle(cuda_device, B, H, Ln, Nc, D):
    """Head dimensions below 128 (68: the reference model's) read natively, with
    the key RMS mean over D."""
    torch = pytest.importorskip("torch")
    from lucid_b200 import decode_update
    from oracle.lucid_oracle import decode_update as ref_update
    g = np.random.default_rng(Nc + D)
    bf = lambda a: (torch.tensor(a, dtype=torch.float32).bfloat16().double().numpy())
    kn, vn = bf(g.standard_normal((B, H, Ln, D))), bf(g.standard_normal((B, H, Ln, D)))
    kc = bf(0.6 * g.standard_normal((B, H, 1, D)) + 0.8 * g.standard_normal((B, H, Nc, D)))
    xc = bf(0.1 * g.standard_normal((B, H, Nc, D)))
    s = D ** -0.5
    ref = ref_update(kn, vn, kc, xc, s, 1e-5)
    x = decode_update(*(_bf(torch, a, cuda_device) for a in (kn, vn, kc, xc)), s, 1e-5).float().cpu().numpy()
    assert x.shape == ref.shape
    err = np.abs(x - ref) - (1e-2 + 2.0 ** -8 * np.abs(ref))
    assert err.max() <= 0, np.abs(x - ref).max()


@pytest.mark.parametrize("B,Hq,Hkv,Ln,Nc,D", [(1, 4, 2, 1, 1000, 128), (2, 2, 2, 3, 300, 128),
                                              (1, 8, 1, 1, 5000, 128), (1, 8, 1, 2, 2000, 68)])
def test_decode_attention_matches_oracle(cuda_device, B, Hq, Hkv, Ln, Nc, D):
    torch = pytest.importorskip("torch")
    from lucid_b200 import decode_attention
    from oracle.lucid_oracle import decode_attention as ref_attn
    g = np.random.default_rng(Nc + Ln)
    bf = lambda a: (torch.tensor(a, dtype=torch.float32).bfloat16().double().numpy())
    q = bf(g.standard_normal((B, Hq, Ln, D)))
    kc = bf(g.standard_normal((B, Hkv, Nc, D)))
    xc = bf(g.standard_normal((B, Hkv, Nc, D)))
    s = D ** -0.5
    ref = ref_attn(q, kc, xc, s)
    o = decode_attention(*(_bf(torch, a, cuda_device) for a in (q, kc, xc)), s).float().cpu().numpy()
    assert o.shape == ref.shape
    err = np.abs(o - ref) - (1e-2 + 2.0 ** -8 * np.abs(ref))
    assert err.max() <= 0, np.abs(o - ref).max()


def _bf16_close(torch, got, ref):
    """|got - ref| <= 1e-2 + 2^-7 |ref|: one bf16 rounding of either side apart."""
    err = (got.float() - ref.float()).abs() - (1e-2 + 2.0 ** -7 * ref.float().abs())
    assert err.max().item() <= 0, (got.float() - ref.float()).abs().max().item()


STEP_CASES = [(4, 8, 8, 1, 5000, 128), (2, 4, 2, 1, 3000, 68), (1, 2, 2, 2, 700, 128), (2, 4, 4, 1, 37, 64),
              (1, 2, 1, 1, 40000, 128)]


@pytest.mark.parametrize("B,Hq,Hkv,Ln,Nc,D", STEP_CASES)
def test_decode_step_matches_two_pass(cuda_device, B, Hq, Hkv, Ln, Nc, D):
    """The fused step (one pass over the cache) against decode_update, the cache
    append and decode_attention (two passes)."""
    torch = pytest.importorskip("torch")
    from lucid_b200 import decode_attention, decode_step, decode_step_fused, decode_update
    assert decode_step_fused(Hq, Hkv, Ln)
    g = torch.Generator(device=cuda_device).manual_seed(Nc + D)
    rn = lambda *sh, sc=1.0: (sc * torch.randn(*sh, generator=g, device=cuda_device)).to(torch.bfloat16)
    q, kn, vn = rn(B, Hq, Ln, D), rn(B, Hkv, Ln, D), rn(B, Hkv, Ln, D)
    kc, xc = rn(B, Hkv, Nc, D), rn(B, Hkv, Nc, D, sc=0.1)
    s = D ** -0.5
    o, x = decode_step(q, kn, vn, kc, xc, s, 1e-5)
    x2 = decode_update(kn, vn, kc, xc, s, 1e-5)
    o2 = decode_attention(q, torch.cat([kc, kn], 2), torch.cat([xc, x2], 2), s)
    assert o.shape == o2.shape == (B, Ln, Hq, D) and x.shape == x2.shape == (B, Hkv, Ln, D)
    _bf16_close(torch, x, x2)
    _bf16_close(torch, o, o2)


@pytest.mark.parametrize("B,Hq,Hkv,Ln,Nc,D", STEP_CASES[:4] + [(1, 2, 2, 2, 0, 128)])
def test_decode_step_matches_oracle(cuda_device, B, Hq, Hkv, Ln, Nc, D):
    """x_new against the oracle's get_new_v_prime and the attention against the
    oracle over the cache with the new tokens appended (x_new rounded to bf16 as
    the cache stores it); an empty cache included."""
    torch = pytest.importorskip("torch")
    from lucid_b200 import decode_step
    from oracle.lucid_oracle import decode_attention as ref_attn
    from oracle.lucid_oracle import decode_update as ref_update
    g = np.random.default_rng(Nc + 7 * Ln)
    bf = lambda a: (torch.tensor(a, dtype=torch.float32).bfloat16().double().numpy())
    q, kn, vn = bf(g.standard_normal((B, Hq, Ln, D))), bf(g.standard_normal((B, Hkv, Ln, D))), \
        bf(g.standard_normal((B, Hkv, Ln, D)))
    kc = bf(0.6 * g.standard_normal((B, Hkv, 1, D)) + 0.8 * g.standard_normal((B, Hkv, Nc, D)))
    xc = bf(0.1 * g.standard_normal((B, Hkv, Nc, D)))
    s = D ** -0.5
    x_ref = ref_update(kn, vn, kc, xc, s, 1e-5)
    o_ref = ref_attn(q, np.concatenate([kc, kn], 2), np.concatenate([xc, bf(x_ref)], 2), s)
    o, x = decode_step(*(_bf(torch, a, cuda_device) for a in (q, kn, vn, kc, xc)), s, 1e-5)
    for got, ref in ((x, x_ref), (o, o_ref)):
        got = got.float().cpu().numpy()
        assert got.shape == ref.shape
        err = np.abs(got - ref) - (1e-2 + 2.0 ** -8 * np.abs(ref))
        assert err.max() <= 0, np.abs(got - ref).max()


@pytest.mark.parametrize("hd,heads,kv", [(128, 4, 2), (68, 4, 2), (68, 8, 1)])
def test_layer_prefill_then_decode_matches_ops(cuda_device, hd, heads, kv):
    """LucidAttention with a cache: prefill fills (raw keys, solved values) and
    a decode step equals decode_update + decode_attention on that cache (head_dim
    128, and the reference model's 68): through the fused step where its shape has
    one (2 query heads per kv head), through the two calls otherwise (8)."""
    torch = pytest.importorskip("torch")
    from transformers import DynamicCache, LlamaConfig
    from lucid_b200 import LucidSolveFunction, decode_attention, decode_step_fused, decode_update
    from lucid_b200.layer import LucidAttention
    torch.manual_seed(0)
    fused = decode_step_fused(heads, kv, 1)
    assert fused == (heads // kv == 2)
    cfg = LlamaConfig(hidden_size=512, num_attention_heads=heads, num_key_value_heads=kv, head_dim=hd,
                      rms_norm_eps=1e-5)
    layer = LucidAttention(cfg, 0).to(cuda_device, torch.bfloat16).eval()
    T = 200
    h = torch.randn(1, T + 1, 512, device=cuda_device, dtype=torch.bfloat16)
    cache = DynamicCache()
    with torch.no_grad():
        layer(h[:, :T], past_key_value=cache)
        out, _ = layer(h[:, T:], past_key_value=cache)
        kc, xc = (cache.layers[0].keys, cache.layers[0].values) if hasattr(cache, "layers") else \
            (cache.key_cache[0], cache.value_cache[0])
        assert kc.shape[2] == T + 1 and xc.shape[2] == T + 1
        # prefill part of the cache holds the solved values
        k_pre = layer.k_proj(h[:, :T]).view(1, T, kv, hd).transpose(1, 2)
        v_pre = layer.v_proj(h[:, :T]).view(1, T, kv, hd).transpose(1, 2)
        x_pre = LucidSolveFunction.apply(k_pre, v_pre, layer.scaling, 1e-5)
        torch.testing.assert_close(xc[:, :, :T], x_pre, rtol=0, atol=0)
        # decode step = decode_update + decode_attention on the cache
        k1 = layer.k_proj(h[:, T:]).view(1, 1, kv, hd).transpose(1, 2)
        v1 = layer.v_proj(h[:, T:]).view(1, 1, kv, hd).transpose(1, 2)
        x1 = decode_update(k1, v1, kc[:, :, :T], xc[:, :, :T], layer.scaling, 1e-5)
        q1 = layer.q_proj(h[:, T:]).view(1, 1, heads, hd).transpose(1, 2)
        o1 = decode_attention(q1, kc, xc, layer.scaling)
        ref = layer.o_proj(o1.reshape(1, 1, -1))
        assert torch.isfinite(out).all()
        if fused:   # one pass, merged in another order: within a bf16 rounding
            _bf16_close(torch, xc[:, :, T:], x1)
            scale = ref.float().abs().max().item()
            assert (out.float() - ref.float()).abs().max().item() <= 1e-2 * scale
        else:       # the same two calls
            torch.testing.assert_close(xc[:, :, T:], x1, rtol=0, atol=0)
            torch.testing.assert_close(out, ref, rtol=0, atol=0)


def _kc_bar(d_k, d_w, d_beta, ref):
    """1e-2, or 1.5x the deviation of the reference's own bf16 key cache
    (oracle/path_precision.py: k_new and the output are bf16 there too)."""
    from oracle.path_precision import reference_bf16_k_cache
    return max(1e-2, 1.5 * float(np.abs(reference_bf16_k_cache(d_k, d_w, d_beta) - ref).max()))


@pytest.mark.parametrize("name", PATH_CASES)
def test_path_key_cache_matches_reference_fixture(cuda_device, name):
    torch = pytest.importorskip("torch")
    from lucid_b200.path import parallel_lucid_path_attention
    d = load_path_golden(name)
    bar = _kc_bar(d["k"], d["w"], d["beta"], d["k_cache"])
    k, v, w, beta = (_bf(torch, d[n], cuda_device) for n in ("k", "v", "w", "beta"))
    q = _bf(torch, d["q"], cuda_device) if d.get("q") is not None else None
    with torch.no_grad():
        o, kc = parallel_lucid_path_attention(k, v, w, beta, q=q, use_cache=True)
    kc = kc.float().cpu().numpy()
    assert np.abs(kc - d["k_cache"]).max() <= bar, (np.abs(kc - d["k_cache"]).max(), bar)


def test_path_key_cache_long_sequence(cuda_device):
    """12 blocks of suffix products against the float64 oracle."""
    torch = pytest.importorskip("torch")
    from lucid_b200.path import parallel_lucid_path_attention
    from oracle.path_oracle import make_path_inputs, path_k_cache
    d = make_path_inputs(8, 1, 1500, 1, 128)
    ref = path_k_cache(d["k"], d["w"], d["beta"])
    k, v, w, beta = (_bf(torch, d[n], cuda_device) for n in ("k", "v", "w", "beta"))
    with torch.no_grad():
        _, kc = parallel_lucid_path_attention(k, v, w, beta, use_cache=True)
    kc = kc.float().cpu().numpy()
    assert np.all(np.isfinite(kc))
    bar = _kc_bar(d["k"], d["w"], d["beta"], ref)
    assert np.abs(kc - ref).max() <= bar, (np.abs(kc - ref).max(), bar)
