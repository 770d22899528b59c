"""Model-facing mirror of the reference layer (modeling_lucid.py:385-618).

``LucidAttention`` keeps the reference's constructor, sub-module names and
method signatures (q/k/v/o projections, ``k_norm``, ``get_v_prime``,
``eager_lucid_attention_forward``, ``create_causal_mask``) so a checkpoint
or a caller written for the reference works unchanged; the attention core
runs on the B200 kernels of lucid_b200.ops.

``patch_reference(module)`` rebinds the two hot methods of an already
imported reference module (its ``LucidAttention`` class) to the B200
kernels, leaving everything else of the reference model untouched.

Training / prefill (past_seq_len == 0) and incremental decoding
(get_new_v_prime, :576-598, then attention over the cache) are both covered;
the cache keeps raw keys and solved values like the reference (:479-481).
Where a single-pass kernel covers the step's shape (ops.decode_step_fused),
``LucidAttention.forward`` computes get_new_v_prime and the attention in one
pass over the cache and then appends to it; the three methods above keep the
reference's separate calls for code that calls or patches them.
"""
from __future__ import annotations

import torch
from torch import nn

from .ops import (LucidAttentionFunction, LucidAttnFunction, LucidSolveFunction, decode_attention, decode_step,
                  decode_step_fused, decode_update)

__all__ = ["LucidAttention", "patch_reference", "get_v_prime", "get_new_v_prime", "eager_lucid_attention_forward"]


def _cache_layer(past_key_value, layer_idx):
    """(keys, values) of one layer of a transformers cache (old key_cache /
    value_cache lists or the layered Cache of transformers 5)."""
    if hasattr(past_key_value, "key_cache"):
        return past_key_value.key_cache[layer_idx], past_key_value.value_cache[layer_idx]
    layer = past_key_value.layers[layer_idx]
    return layer.keys, layer.values


def _k_norm_eps(self) -> float:
    eps = getattr(self.k_norm, "eps", None)
    return float(eps) if eps is not None else 1e-5


def get_v_prime(self, key: torch.Tensor, value: torch.Tensor, scaling: float,
                attention_mask: torch.Tensor | None = None) -> torch.Tensor:
    """X = P^-1 V with P = tril(exp(s k_norm(K) k_norm(K)^T - 1/s))
    (modeling_lucid.py:551-574).  ``attention_mask`` is accepted for
    signature compatibility; the kernels apply the causal structure by index
    arithmetic.  Both the dense (N < 2^16) and the blockwise (N >= 2^16,
    Lucid_Tril_Solver) branches of the reference map to the same kernel."""
    which = getattr(self, "which_rmsnorm", "exp_k_norm")
    if which != "exp_k_norm":
        raise NotImplementedError(f"{which} not implemented")
    return LucidSolveFunction.apply(key, value, float(scaling), _k_norm_eps(self))


def get_new_v_prime(self, key: torch.Tensor, value: torch.Tensor, attention_mask: torch.Tensor | None,
                    scaling: float, past_key_value) -> torch.Tensor:
    """Decode step (modeling_lucid.py:576-598): x_new = value -
    exp(s k_norm(key) k_norm(K_cache)^T - 1/s) X_cache, one pass over the cache on
    the B200 (cached keys normalised on the fly)."""
    which = getattr(self, "which_rmsnorm", "exp_k_norm")
    if which != "exp_k_norm":
        raise NotImplementedError(f"{which} not implemented")
    k_cache, x_cache = _cache_layer(past_key_value, self.layer_idx)
    return decode_update(key, value, k_cache, x_cache, float(scaling), _k_norm_eps(self))


def eager_lucid_attention_forward(self, query: torch.Tensor, key: torch.Tensor, v_prime: torch.Tensor,
                                  scaling: float, attention_mask: torch.Tensor | None = None, **kwargs):
    """softmax(scaling Q K^T + causal) repeat_kv(X), returned as
    (O [B, N, Hq, D], None) like modeling_lucid.py:505-549.  Grouped-query
    heads are handled natively (no repeat_kv copy).  With fewer queries than
    keys (decoding against a cache) the queries sit at the end of the key
    sequence, as the reference's causal mask places them (:600-618)."""
    if query.shape[-2] != key.shape[-2]:
        return decode_attention(query, key, v_prime, float(scaling)), None
    return LucidAttnFunction.apply(query, key, v_prime, float(scaling)), None


class LucidAttention(nn.Module):
    """LUCID attention layer (modeling_lucid.py:385-503) on B200 kernels."""

    def __init__(self, config, layer_idx: int):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.head_dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
        self.num_key_value_groups = config.num_attention_heads // config.num_key_value_heads
        self.scaling = self.head_dim ** -0.5
        self.attention_dropout = getattr(config, "attention_dropout", 0.0)
        self.is_causal = True
        self.use_rope = getattr(config, "use_rope", False)
        self.which_rmsnorm = getattr(config, "which_rmsnorm", "exp_k_norm")
        bias = getattr(config, "attention_bias", False)
        self.q_proj = nn.Linear(config.hidden_size, config.num_attention_heads * self.head_dim, bias=bias)
        self.k_proj = nn.Linear(config.hidden_size, config.num_key_value_heads * self.head_dim, bias=bias)
        self.v_proj = nn.Linear(config.hidden_size, config.num_key_value_heads * self.head_dim, bias=bias)
        if self.which_rmsnorm != "exp_k_norm":
            raise NotImplementedError(f"{self.which_rmsnorm} not implemented")
        self.k_norm = nn.RMSNorm(self.head_dim, eps=getattr(config, "rms_norm_eps", 1e-5),
                                 elementwise_affine=False)
        self.o_proj = nn.Linear(config.num_attention_heads * self.head_dim, config.hidden_size, bias=bias)

    get_v_prime = get_v_prime
    get_new_v_prime = get_new_v_prime
    eager_lucid_attention_forward = eager_lucid_attention_forward

    def create_causal_mask(self, query, key, past_seq_len: int, attention_mask=None):
        """(B, 1, Lq, Lq + past) boolean causal mask (modeling_lucid.py:600-618);
        kept for callers, not used by the kernels."""
        b, _, lq, _ = query.shape
        tot = lq + past_seq_len
        qi = torch.arange(lq, device=query.device)
        ki = torch.arange(tot, device=query.device)
        m = (ki[None, :] <= (qi[:, None] + past_seq_len))[None, None].expand(b, 1, -1, -1)
        if attention_mask is not None:
            m = m & attention_mask.reshape(m.shape)
        return m

    def forward(self, hidden_states: torch.Tensor, position_embeddings=None, attention_mask=None,
                past_key_value=None, cache_position=None, **kwargs):
        """modeling_lucid.py:421-503: projections, LUCID attention, o_proj.  Without
        a cache (training) the fused op runs; with a cache the prefill solves X,
        decoding steps use get_new_v_prime, and the cache is updated with raw keys
        and solved values before the attention, as in the reference."""
        if self.use_rope:
            raise NotImplementedError("use_rope=True is not supported by this layer")
        input_shape = hidden_states.shape[:-1]
        hidden_shape = (*input_shape, -1, self.head_dim)
        q = self.q_proj(hidden_states).view(hidden_shape).transpose(1, 2)
        k = self.k_proj(hidden_states).view(hidden_shape).transpose(1, 2)
        v = self.v_proj(hidden_states).view(hidden_shape).transpose(1, 2)
        if past_key_value is None or self.training:
            o = LucidAttentionFunction.apply(q, k, v, float(self.scaling), float(self.k_norm.eps or 1e-5))
        else:
            past = past_key_value.get_seq_length(self.layer_idx)
            o = None
            if past == 0:
                x = self.get_v_prime(k, v, self.scaling, None)
            elif decode_step_fused(q.shape[1], k.shape[1], k.shape[2]):
                # get_new_v_prime and the attention in one pass over the cache
                k_cache, x_cache = _cache_layer(past_key_value, self.layer_idx)
                o, x = decode_step(q, k, v, k_cache, x_cache, float(self.scaling), _k_norm_eps(self))
            else:
                x = self.get_new_v_prime(k, v, None, self.scaling, past_key_value)
            k_all, x_all = past_key_value.update(k, x, self.layer_idx,
                                                 {"cache_position": cache_position})
            if o is None:
                o, _ = self.eager_lucid_attention_forward(q, k_all, x_all, self.scaling, None)
        o = o.reshape(*input_shape, -1).contiguous()
        return self.o_proj(o), None


def patch_reference(module) -> None:
    """Rebind ``module.LucidAttention.get_v_prime``, ``.get_new_v_prime`` and
    ``.eager_lucid_attention_forward`` (an imported modeling_lucid module)
    to the B200 kernels."""
    cls = module.LucidAttention
    cls.get_v_prime = get_v_prime
    cls.get_new_v_prime = get_new_v_prime
    cls.eager_lucid_attention_forward = eager_lucid_attention_forward
