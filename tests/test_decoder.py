"""The Llama-architecture decoder with LUCID attention (lucid_b200/decoder.py),
the reference model of lucid/config/config.json, for the full-model prefill.

CPU: the configuration and the parameter count of the full model (built on
the meta device).  GPU: a small model with the reference's head_dim 68 and
8 query heads per kv head against a float32 torch restatement of the same
model (attention by oracle/torch_ref.py, the reference's own torch path), and
the cache-filling prefill against the fused one."""
import pytest
import torch

from conftest import ROOT  # noqa: F401  (puts the repo on sys.path)


def test_config_matches_reference_model():
    from lucid_b200.decoder import LucidForCausalLM, lucid_config
    cfg = lucid_config()
    assert (cfg.hidden_size, cfg.intermediate_size, cfg.num_hidden_layers) == (2048, 5632, 22)
    assert (cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim, cfg.vocab_size) == (32, 4, 68, 32000)
    assert cfg.use_rope is False and cfg.which_rmsnorm == "exp_k_norm"
    with torch.device("meta"):
        m = LucidForCausalLM(cfg)
    per_layer = (2048 * 32 * 68 + 2 * 2048 * 4 * 68 + 32 * 68 * 2048) + 3 * 2048 * 5632 + 2 * 2048
    expect = 2 * 32000 * 2048 + 22 * per_layer + 2048
    assert sum(p.numel() for p in m.parameters()) == expect


def _ref_forward(model, ids, eps=1e-5):
    """float32 restatement of LucidForCausalLM.forward: LlamaRMSNorm, projections,
    the reference's LUCID attention (torch_ref.lucid_layer), SiLU MLP."""
    from oracle import torch_ref
    cfg = model.config
    hd, hq, hk = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    W = {n: p.detach().float() for n, p in model.named_parameters()}

    def norm(x, w):
        return w * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps))

    x = W["embed_tokens.weight"][ids]
    B, N, _ = x.shape
    for i in range(cfg.num_hidden_layers):
        p = f"layers.{i}."
        h = norm(x, W[p + "input_layernorm.weight"])
        q = (h @ W[p + "self_attn.q_proj.weight"].T).view(B, N, hq, hd).transpose(1, 2)
        k = (h @ W[p + "self_attn.k_proj.weight"].T).view(B, N, hk, hd).transpose(1, 2)
        v = (h @ W[p + "self_attn.v_proj.weight"].T).view(B, N, hk, hd).transpose(1, 2)
        o = torch_ref.lucid_layer(q, k, v, hd ** -0.5, eps).reshape(B, N, hq * hd)
        x = x + o @ W[p + "self_attn.o_proj.weight"].T
        h = norm(x, W[p + "post_attention_layernorm.weight"])
        g = torch.nn.functional.silu(h @ W[p + "mlp.gate_proj.weight"].T) * (h @ W[p + "mlp.up_proj.weight"].T)
        x = x + g @ W[p + "mlp.down_proj.weight"].T
    return norm(x, W["norm.weight"]) @ W["lm_head.weight"].T


@pytest.mark.gpu
def test_small_decoder_matches_torch_restatement(cuda_device):
    from transformers import DynamicCache

    from lucid_b200.decoder import LucidForCausalLM, lucid_config
    cfg = lucid_config(hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=8,
                       num_key_value_heads=1, head_dim=68, vocab_size=1000)
    model = LucidForCausalLM(cfg).to(cuda_device, torch.bfloat16).init_weights(seed=3, std=0.05).eval()
    g = torch.Generator().manual_seed(4)
    ids = torch.randint(0, cfg.vocab_size, (2, 384), generator=g).to(cuda_device)
    with torch.no_grad():
        fused = model(ids).float()
        cache = DynamicCache()
        cached = model(ids, past_key_values=cache).float()
        last = model(ids, logits_to_keep=1).float()
    ref = _ref_forward(model, ids)
    scale = ref.abs().max().item()
    assert torch.isfinite(fused).all()
    assert (fused - ref).abs().max().item() <= 3e-2 * scale, (fused - ref).abs().max().item() / scale
    # the cache-filling prefill (solve, cache update, attention) computes the same logits
    assert (cached - fused).abs().max().item() <= 1e-2 * scale
    torch.testing.assert_close(last, fused[:, -1:], rtol=0, atol=0)
    assert cache.get_seq_length(0) == 384
