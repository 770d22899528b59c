"""lucid_b200 — LUCID attention on B200 (sm_100a) tensor-core kernels.

    from lucid_b200 import lucid_attention
    o = lucid_attention(q, k, v)          # q [B,Hq,N,128], k/v [B,Hkv,N,128] bf16

The model-facing mirror of the reference layer is lucid_b200.layer.LucidAttention.
"""
from .ops import (  # noqa: F401
    LucidAttentionFunction,
    LucidAttnFunction,
    LucidSolveFunction,
    attn_bwd,
    attn_fwd,
    fused_fwd,
    decode_attention,
    decode_step,
    decode_step_fused,
    decode_update,
    lucid_attention,
    padded_len,
    solve_bwd,
    solve_fwd,
)

__version__ = "0.1.0"
