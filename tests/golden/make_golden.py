"""Generate the golden LUCID fixtures from the reference implementation.

Runs the reference's own PyTorch path (modeling_lucid.py of
saisuryadv/LUCID, loaded from a local checkout) in float64 on the CPU and
stores inputs and outputs as compressed .npz files next to this script:

  LucidAttention.get_v_prime            (modeling_lucid.py:551-574)
  LucidAttention.eager_lucid_attention_forward (modeling_lucid.py:505-549)
  Lucid_Tril_Solver.apply (blockwise)   (modeling_lucid.py:284-382)
  torch.autograd for dQ, dK, dV

Inputs are rounded to bf16-representable values (stored as float32) so the
same fixture drives the bf16 GPU kernels.  The reference checkout is only
needed to regenerate; the fixtures themselves are committed.

It also stores ``decode_*.npz``: LucidAttention.get_new_v_prime
(modeling_lucid.py:576-598) for one decode step against a key / value cache.

Usage:  python tests/golden/make_golden.py /path/to/LUCID [--decode-only]
"""
from __future__ import annotations

import importlib.util
import os
import sys
import typing

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(root: str):
    import transformers
    import transformers.utils

    # transformers 5.x removed LossKwargs, which modeling_lucid.py imports.
    if not hasattr(transformers.utils, "LossKwargs"):
        class LossKwargs(typing.TypedDict, total=False):
            pass
        transformers.utils.LossKwargs = LossKwargs
    name = "transformers.models.llama.modeling_lucid"
    spec = importlib.util.spec_from_file_location(name, os.path.join(root, "modeling_lucid.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def bf16_round(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(torch.float64)


def make_inputs(seed: int, B: int, Hq: int, Hkv: int, N: int, D: int, keys: str = "iid",
                q_scale: float = 1.0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, N, D, generator=g, dtype=torch.float64) * q_scale
    if keys == "iid":
        k = torch.randn(B, Hkv, N, D, generator=g, dtype=torch.float64)
    else:  # correlated keys K = 0.6 s + 0.8 n (long-context stress distribution)
        s = torch.randn(B, Hkv, 1, D, generator=g, dtype=torch.float64)
        n = torch.randn(B, Hkv, N, D, generator=g, dtype=torch.float64)
        k = 0.6 * s + 0.8 * n
    v = torch.randn(B, Hkv, N, D, generator=g, dtype=torch.float64)
    do = torch.randn(B, N, Hq, D, generator=g, dtype=torch.float64)
    return [bf16_round(t) for t in (q, k, v, do)]


def reference_case(mod, q, k, v, do, eps: float = 1e-5):
    from transformers import LlamaConfig

    B, Hq, N, D = q.shape
    Hkv = k.shape[1]
    cfg = LlamaConfig(hidden_size=Hq * D, num_attention_heads=Hq, num_key_value_heads=Hkv,
                      head_dim=D, rms_norm_eps=eps, attention_bias=False)
    cfg.use_rope = False
    att = mod.LucidAttention(cfg, 0).double()
    att.train()
    q = q.clone().requires_grad_(True)
    k = k.clone().requires_grad_(True)
    v = v.clone().requires_grad_(True)
    mask = att.create_causal_mask(q, k, 0)
    x = att.get_v_prime(k, v, att.scaling, mask)
    o, _ = att.eager_lucid_attention_forward(q, k, x, att.scaling, mask)
    (o * do).sum().backward()
    return dict(o=o.detach().numpy(), x=x.detach().numpy(), dq=q.grad.numpy(), dk=k.grad.numpy(),
                dv=v.grad.numpy(), scale=np.float64(att.scaling), eps=np.float64(eps))


def blockwise_case(mod, k, v, dx, bs: int, eps: float = 1e-5):
    """Lucid_Tril_Solver forward + backward (inputs: normalised keys)."""
    D = k.shape[-1]
    scale = D ** -0.5
    khat = torch.nn.functional.rms_norm(k, (D,), eps=eps).detach().requires_grad_(True)
    vv = v.clone().requires_grad_(True)
    x = mod.Lucid_Tril_Solver.apply(khat, vv.clone(), scale, bs)  # forward mutates its value arg
    (x * dx).sum().backward()
    return dict(khat=khat.detach().numpy(), x=x.detach().numpy(), dkhat=khat.grad.numpy(),
                dv=vv.grad.numpy(), dx=dx.numpy(), scale=np.float64(scale), bs=np.int64(bs))


def decode_case(mod, B: int, H: int, Nc: int, Ln: int, D: int, seed: int, eps: float = 1e-5):
    """LucidAttention.get_new_v_prime (modeling_lucid.py:576-598): one decode step
    against a cache of raw keys and solved values (the cache convention of :479-481)."""
    from transformers import LlamaConfig
    cfg = LlamaConfig(hidden_size=H * D, num_attention_heads=H, num_key_value_heads=H, head_dim=D,
                      rms_norm_eps=eps, attention_bias=False)
    cfg.use_rope = False
    att = mod.LucidAttention(cfg, 0).double()
    g = torch.Generator().manual_seed(seed)
    kc = bf16_round(torch.randn(B, H, Nc, D, generator=g, dtype=torch.float64))
    xc = bf16_round(torch.randn(B, H, Nc, D, generator=g, dtype=torch.float64))
    kn = bf16_round(torch.randn(B, H, Ln, D, generator=g, dtype=torch.float64))
    vn = bf16_round(torch.randn(B, H, Ln, D, generator=g, dtype=torch.float64))

    class Cache:  # the two attributes get_new_v_prime reads
        key_cache = [kc]
        value_cache = [xc]

    with torch.no_grad():
        x = att.get_new_v_prime(kn, vn, None, att.scaling, past_key_value=Cache())
    return dict(x_new=x.numpy().astype(np.float32), k_cache_bf16=bf16_bits(kc.numpy()),
                x_cache_bf16=bf16_bits(xc.numpy()), k_new_bf16=bf16_bits(kn.numpy()),
                v_new_bf16=bf16_bits(vn.numpy()), scale=np.float64(att.scaling), eps=np.float64(eps))


def f32(d):
    return {kk: (vv.astype(np.float32) if isinstance(vv, np.ndarray) and vv.dtype == np.float64 else vv)
            for kk, vv in d.items()}


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """Exact bf16 values (already rounded) -> their uint16 bit patterns."""
    return (np.ascontiguousarray(a, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


CASES = [
    # name, seed, B, Hq, Hkv, N, D, keys, q_scale
    ("mha_small_d32", 1, 1, 2, 2, 48, 32, "iid", 1.0),
    ("gqa_ragged_d128", 2, 1, 4, 2, 130, 128, "iid", 1.0),
    ("stress_d128", 3, 1, 1, 1, 256, 128, "corr", 1.0),
    ("cfg2_like_d128", 4, 2, 1, 1, 136, 128, "iid", 128 ** -0.5),
]


DECODE_CASES = {
    # name: (B, H, cache length, new tokens, D, seed)
    "decode_d128": (1, 2, 300, 1, 128, 11),
    "decode_multi_d128": (2, 1, 777, 3, 128, 12),
}


def main(argv):
    root = argv[1] if len(argv) > 1 else os.environ.get("LUCID_REFERENCE", "")
    if not root or not os.path.exists(os.path.join(root, "modeling_lucid.py")):
        print("usage: make_golden.py /path/to/LUCID (checkout containing modeling_lucid.py)")
        return 2
    torch.manual_seed(0)
    mod = load_reference(root)
    for name, (B, H, Nc, Ln, D, seed) in DECODE_CASES.items():
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **decode_case(mod, B, H, Nc, Ln, D, seed))
        print("wrote", name)
    if "--decode-only" in argv:
        return 0
    for name, seed, B, Hq, Hkv, N, D, keys, qs in CASES:
        q, k, v, do = make_inputs(seed, B, Hq, Hkv, N, D, keys, qs)
        out = reference_case(mod, q, k, v, do)
        out = f32(out)
        out.update({f"{nm}_bf16": bf16_bits(t.numpy()) for nm, t in (("q", q), ("k", k), ("v", v), ("do", do))})
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
        print("wrote", name, {kk: getattr(vv, "shape", vv) for kk, vv in out.items()})
    # blockwise solver (Lucid_Tril_Solver) with a small block size
    g = torch.Generator().manual_seed(7)
    k = bf16_round(torch.randn(1, 2, 64, 16, generator=g, dtype=torch.float64))
    v = bf16_round(torch.randn(1, 2, 64, 16, generator=g, dtype=torch.float64))
    dx = bf16_round(torch.randn(1, 2, 64, 16, generator=g, dtype=torch.float64))
    out = blockwise_case(mod, k, v, dx, bs=16)
    out.update(k=k.numpy(), v=v.numpy())
    np.savez_compressed(os.path.join(HERE, "blockwise_bs16.npz"), **out)
    print("wrote blockwise_bs16")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
