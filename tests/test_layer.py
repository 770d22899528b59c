"""The model-facing mirror of the reference layer (lucid_b200/layer.py)."""
import types

import numpy as np
import pytest
import torch

from lucid_b200 import layer as L


def _cfg(hq=4, hkv=2, d=128):
    return types.SimpleNamespace(hidden_size=hq * d, num_attention_heads=hq, num_key_value_heads=hkv,
                                 head_dim=d, rms_norm_eps=1e-5, attention_bias=False, use_rope=False,
                                 attention_dropout=0.0)


def test_layer_mirrors_reference_structure():
    att = L.LucidAttention(_cfg(), 0)
    assert att.scaling == 128 ** -0.5
    assert att.num_key_value_groups == 2
    names = {n for n, _ in att.named_modules()}
    assert {"q_proj", "k_proj", "v_proj", "o_proj", "k_norm"} <= names
    m = att.create_causal_mask(torch.zeros(2, 4, 5, 128), None, 0)
    assert m.shape == (2, 1, 5, 5) and bool(m[0, 0, 4, 0]) and not bool(m[0, 0, 0, 4])


def test_patch_reference_rebinds_hot_methods():
    class FakeLucidAttention:
        def get_v_prime(self, *a, **k):
            return "ref"

        def eager_lucid_attention_forward(self, *a, **k):
            return "ref"

    mod = types.SimpleNamespace(LucidAttention=FakeLucidAttention)
    L.patch_reference(mod)
    assert FakeLucidAttention.get_v_prime is L.get_v_prime
    assert FakeLucidAttention.eager_lucid_attention_forward is L.eager_lucid_attention_forward


@pytest.mark.gpu
def test_layer_forward_backward_matches_oracle(cuda_device):
    from oracle import lucid_oracle as orc
    torch.manual_seed(0)
    att = L.LucidAttention(_cfg(), 0).to(cuda_device, torch.bfloat16)
    h = torch.randn(1, 200, 512, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
    y, _ = att(h)
    y.float().square().mean().backward()
    torch.cuda.synchronize()
    # oracle: same bf16 projections, attention core in float64
    with torch.no_grad():
        hs = (1, 200, -1, 128)
        q = att.q_proj(h).view(hs).transpose(1, 2).double().cpu().numpy()
        k = att.k_proj(h).view(hs).transpose(1, 2).double().cpu().numpy()
        v = att.v_proj(h).view(hs).transpose(1, 2).double().cpu().numpy()
    o, _ = orc.lucid_fwd(q, k, v, 128 ** -0.5)
    o_t = torch.as_tensor(o.reshape(1, 200, -1)).to(cuda_device, torch.bfloat16)
    y_ref = att.o_proj(o_t)
    err = (y.float() - y_ref.float()).abs().max().item()
    assert err < 2e-2, err
    assert torch.isfinite(h.grad).all()
