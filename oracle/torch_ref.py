"""Reference LUCID path restated in PyTorch — TEST / BASELINE INFRASTRUCTURE.

Used only by bench.py (the timed CPU baseline and the `--impl reference`
arm) and by tests.  It restates, op for op, the reference's training path
for one LUCID attention layer (saisuryadv/LUCID modeling_lucid.py):

  get_v_prime (:551-574):      k_norm(key); einsum("bhld,bhsd->bhls");
                               mul_(s).sub_(1/s); masked_fill_(~mask, -inf);
                               exp_(); torch.linalg.solve_triangular(upper=False)
  create_causal_mask (:600-618)
  eager_lucid_attention_forward (:505-549): SDPA(q, repeat_kv(k), repeat_kv(x),
                               is_causal=True, scale=s), transpose(1, 2)
  backward: torch autograd, as in the reference's training step.

The reference module itself cannot be imported on the GPU box (it needs a
transformers fork and is not shipped there), so this restatement is the
"port" CPU baseline.  tests/test_oracle_torch.py checks it against the
golden fixtures made from the real module.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def causal_mask(q: torch.Tensor, past: int = 0) -> torch.Tensor:
    b, _, lq, _ = q.shape
    tot = lq + past
    qi = torch.arange(lq, device=q.device)
    ki = torch.arange(tot, device=q.device)
    m = ki[None, :] <= (qi[:, None] + past)
    return m[None, None].expand(b, 1, -1, -1)


def repeat_kv(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    if n_rep == 1:
        return x
    b, h, n, d = x.shape
    return x[:, :, None].expand(b, h, n_rep, n, d).reshape(b, h * n_rep, n, d)


def get_v_prime(key, value, scaling: float, mask, eps: float = 1e-5):
    key = F.rms_norm(key, (key.shape[-1],), eps=eps)
    s = torch.einsum("bhld,bhsd->bhls", key, key)
    s.mul_(scaling).sub_(1 / scaling)
    s.masked_fill_(~mask[:, :, :, : key.shape[-2]], float("-inf"))
    s.exp_()
    return torch.linalg.solve_triangular(s, value, upper=False)


def lucid_layer(q, k, v, scaling: float | None = None, eps: float = 1e-5):
    """O [B, N, Hq, D] = eager_lucid_attention_forward(q, k, get_v_prime(k, v))."""
    if scaling is None:
        scaling = q.shape[-1] ** -0.5
    mask = causal_mask(q)
    x = get_v_prime(k, v, scaling, mask, eps)
    g = q.shape[1] // k.shape[1]
    o = F.scaled_dot_product_attention(q, repeat_kv(k, g), repeat_kv(x, g), dropout_p=0.0,
                                       scale=scaling, is_causal=True)
    return o.transpose(1, 2).contiguous()


def lucid_fwd_bwd(q, k, v, do, scaling: float | None = None, eps: float = 1e-5):
    """One training step of the layer: forward, then backward with dO."""
    q = q.detach().requires_grad_(True)
    k = k.detach().requires_grad_(True)
    v = v.detach().requires_grad_(True)
    o = lucid_layer(q, k, v, scaling, eps)
    o.backward(do)
    return o.detach(), q.grad, k.grad, v.grad
