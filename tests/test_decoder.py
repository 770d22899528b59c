"""The Llama-architecture decoder with LUCID attention (lucid_b200/decoder.py),
the reference model of lucid/config/config.json, for the full-model prefill.

CPU: the configuration and the parameter count of the full model (built on
the meta device), and loading a reference checkpoint's state dict.  GPU: a small model with the reference's head_dim 68 and
8 query heads per kv head against a float32 torch restatement of the same
model (attention by oracle/torch_ref.py, the reference's own torch path): the
prefill logits, the cache-filling prefill against the fused one, and one
training step's parameter gradients (the LUCID backward inside the model)."""
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


def test_reference_state_dict_loads():
    """A checkpoint saved from the reference's LlamaForCausalLM (``model.`` prefix,
    lm_head at the top) loads with every parameter in place."""
    from lucid_b200.decoder import LucidForCausalLM, lucid_config
    cfg = lucid_config(hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                       num_key_value_heads=2, head_dim=16, vocab_size=50)
    src = LucidForCausalLM(cfg).init_weights(seed=1)
    ref_sd = {(k if k.startswith("lm_head.") else "model." + k): v for k, v in src.state_dict().items()}
    ref_sd["model.rotary_emb.inv_freq"] = torch.ones(8)
    assert "model.layers.1.self_attn.k_proj.weight" in ref_sd and "model.norm.weight" in ref_sd
    dst = LucidForCausalLM(cfg).init_weights(seed=2)
    dst.load_reference_state_dict(ref_sd)
    for (n, a), (_, b) in zip(src.named_parameters(), dst.named_parameters()):
        assert torch.equal(a, b), n


def _ref_forward(model, ids, eps=1e-5):
    """float32 restatement of LucidForCausalLM.forward: LlamaRMSNorm, projections,
    the reference's LUCID attention (torch_ref.lucid_layer), SiLU MLP."""
    from oracle import torch_ref
    cfg = model.config
    hd, hq, hk = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    # float32 parameters are used as they are (a training-step reference differentiates
    # through them); the bf16 model's are copied to float32
    W = {n: p if p.dtype == torch.float32 else p.detach().float() for n, p in model.named_parameters()}

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


@pytest.mark.gpu
def test_small_decoder_training_step_gradients(cuda_device):
    """Next-token cross-entropy through the whole model; every parameter gradient
    against autograd through the float32 restatement (relative L2 error)."""
    from lucid_b200.decoder import LucidForCausalLM, lucid_config
    cfg = lucid_config(hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=8,
                       num_key_value_heads=1, head_dim=68, vocab_size=1000)
    model = LucidForCausalLM(cfg).to(cuda_device, torch.bfloat16).init_weights(seed=5, std=0.05).train()
    g = torch.Generator().manual_seed(6)
    ids = torch.randint(0, cfg.vocab_size, (2, 300), generator=g).to(cuda_device)
    logits = model(ids)
    loss = torch.nn.functional.cross_entropy(logits[:, :-1].float().reshape(-1, cfg.vocab_size),
                                             ids[:, 1:].reshape(-1))
    loss.backward()
    ref_params = {n: p.detach().float().clone().requires_grad_(True) for n, p in model.named_parameters()}

    class _View:   # the restatement reads weights by name
        config = cfg

        def named_parameters(self):
            return ref_params.items()
    ref_logits = _ref_forward(_View(), ids)
    ref_loss = torch.nn.functional.cross_entropy(ref_logits[:, :-1].reshape(-1, cfg.vocab_size), ids[:, 1:].reshape(-1))
    ref_loss.backward()
    assert abs(loss.item() - ref_loss.item()) < 1e-2 * abs(ref_loss.item())
    worst = {}
    for n, p in model.named_parameters():
        gr = ref_params[n].grad
        assert p.grad is not None and torch.isfinite(p.grad).all(), n
        worst[n] = ((p.grad.float() - gr).norm() / gr.norm().clamp_min(1e-30)).item()
    bad = {n: e for n, e in worst.items() if e > 5e-2}
    assert not bad, bad
