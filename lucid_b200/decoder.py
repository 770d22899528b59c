"""Llama-architecture decoder with LUCID attention on the B200 kernels: the
reference's model (modeling_lucid.py: LlamaMLP :155-168, LlamaDecoderLayer
:621-684, LlamaModel.forward :741-846, LlamaForCausalLM :847-968) for
prefill, with the hyperparameters of its lucid/config/config.json.

Only the attention runs on this package's kernels (layer.LucidAttention:
the fused solve + attention without a cache, or get_v_prime + cache fill +
attention with one, as the reference's prefill does with use_cache=True).
Embedding, RMSNorm, the SiLU MLP and the LM head are stock torch modules
(cuBLAS GEMMs): they are not part of the accelerated path.

Reference configuration notes:
  * head_dim 68 (> hidden / heads = 64): the attention kernels run it
    zero-padded to 128 columns with the key RMS mean over 68 (ops.py);
  * use_rope false (NoPE), which_rmsnorm "exp_k_norm";
  * use_beta true: the reference computes beta from a beta_proj that its
    LucidAttention never defines and never uses beta in the attention, so
    beta has no effect on the model's math and is not built here;
  * attention_type "oglucid", which the reference's LlamaDecoderLayer
    rejects (it accepts "lucid" / "llama"): every layer is LUCID here.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from .layer import LucidAttention

__all__ = ["LUCID_CONFIG", "lucid_config", "LucidRMSNorm", "LucidMLP", "LucidDecoderLayer", "LucidForCausalLM"]

# lucid/config/config.json (the fields the model's math depends on)
LUCID_CONFIG = dict(
    hidden_size=2048, intermediate_size=5632, num_hidden_layers=22, num_attention_heads=32,
    num_key_value_heads=4, head_dim=68, vocab_size=32000, rms_norm_eps=1e-5, hidden_act="silu",
    attention_bias=False, mlp_bias=False, tie_word_embeddings=False, initializer_range=0.02,
    use_rope=False, which_rmsnorm="exp_k_norm", bos_token_id=1, eos_token_id=2,
)


def lucid_config(**overrides):
    """A transformers LlamaConfig with the reference model's hyperparameters
    (any field overridable, e.g. num_hidden_layers for a smaller model)."""
    from transformers import LlamaConfig
    kw = dict(LUCID_CONFIG)
    kw.update(overrides)
    extra = {k: kw.pop(k) for k in ("use_rope", "which_rmsnorm")}
    cfg = LlamaConfig(**kw)
    for k, v in extra.items():
        setattr(cfg, k, v)
    return cfg


class LucidRMSNorm(nn.Module):
    """LlamaRMSNorm: weight * (x / sqrt(mean(x^2) + eps)) computed in fp32."""

    def __init__(self, hidden_size: int, eps: float = 1e-5):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.eps = eps

    def forward(self, x):
        dt = x.dtype
        h = x.float()
        h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + self.eps)
        return self.weight * h.to(dt)


class LucidMLP(nn.Module):
    def __init__(self, config):
        super().__init__()
        bias = getattr(config, "mlp_bias", False)
        self.gate_proj = nn.Linear(config.hidden_size, config.intermediate_size, bias=bias)
        self.up_proj = nn.Linear(config.hidden_size, config.intermediate_size, bias=bias)
        self.down_proj = nn.Linear(config.intermediate_size, config.hidden_size, bias=bias)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class LucidDecoderLayer(nn.Module):
    """Pre-norm residual block: x + attn(norm(x)), then x + mlp(norm(x))."""

    def __init__(self, config, layer_idx: int):
        super().__init__()
        self.self_attn = LucidAttention(config, layer_idx)
        self.mlp = LucidMLP(config)
        self.input_layernorm = LucidRMSNorm(config.hidden_size, config.rms_norm_eps)
        self.post_attention_layernorm = LucidRMSNorm(config.hidden_size, config.rms_norm_eps)

    def forward(self, x, past_key_value=None, attn_events=None):
        h = self.input_layernorm(x)
        if attn_events is not None:
            attn_events[0].record()
        h, _ = self.self_attn(h, past_key_value=past_key_value)
        if attn_events is not None:
            attn_events[1].record()
        x = x + h
        return x + self.mlp(self.post_attention_layernorm(x))


class LucidForCausalLM(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.config = config
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList(LucidDecoderLayer(config, i) for i in range(config.num_hidden_layers))
        self.norm = LucidRMSNorm(config.hidden_size, config.rms_norm_eps)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)

    @torch.no_grad()
    def init_weights(self, seed: int = 0, std: float | None = None):
        """Normal(0, initializer_range) for every linear and embedding weight,
        ones for the norms (LlamaPreTrainedModel._init_weights)."""
        std = self.config.initializer_range if std is None else std
        g = torch.Generator(device=self.lm_head.weight.device).manual_seed(seed)
        for m in self.modules():
            if isinstance(m, (nn.Linear, nn.Embedding)):
                m.weight.copy_(torch.randn(m.weight.shape, generator=g, device=m.weight.device) * std)
                if getattr(m, "bias", None) is not None:
                    m.bias.zero_()
            elif isinstance(m, LucidRMSNorm):
                m.weight.fill_(1.0)
        return self

    def load_reference_state_dict(self, state_dict, strict: bool = True):
        """Load a state dict of the reference's LlamaForCausalLM (modeling_lucid.py:847-968:
        ``model.embed_tokens.weight``, ``model.layers.{i}.self_attn.q_proj.weight`` …,
        ``model.norm.weight``, ``lm_head.weight``).  The submodule names are the
        reference's, so only the ``model.`` prefix goes; rotary ``inv_freq`` buffers
        (non-persistent in the reference, unused by this NoPE model) are skipped if a
        checkpoint carries them."""
        sd = {}
        for k, v in state_dict.items():
            if k.endswith("rotary_emb.inv_freq"):
                continue
            sd[k[len("model."):] if k.startswith("model.") else k] = v
        return self.load_state_dict(sd, strict=strict)

    def forward(self, input_ids, past_key_values=None, logits_to_keep: int = 0, attn_events=None):
        """Logits of the last ``logits_to_keep`` positions (0: all).  With a
        transformers Cache, the prefill fills it (raw keys, solved values) as
        the reference does.  attn_events: optional per-layer pairs of CUDA
        events recorded around each attention call."""
        x = self.embed_tokens(input_ids)
        for i, layer in enumerate(self.layers):
            x = layer(x, past_key_value=past_key_values,
                      attn_events=None if attn_events is None else attn_events[i])
        x = self.norm(x)
        if logits_to_keep:
            x = x[:, -logits_to_keep:]
        return self.lm_head(x)
