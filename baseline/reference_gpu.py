"""The reference's own GPU code, run as a comparator by bench.py (measurement only).

Nothing in lucid_b200 imports this module.  It loads the unmodified reference files
that baseline/install_ref.py copied into baseline/_ref/ and times them on the same
GPU, on the same seeded inputs as our kernels, and measures how far they and we
are from the float32 / float64 results the parity tests use:

  torch path (config 2)   LucidAttention.get_v_prime (modeling_lucid.py:551-574) and
                          eager_lucid_attention_forward (:505-549, SDPA), forward and
                          autograd backward.  torch.linalg.solve_triangular has no
                          bf16 CUDA kernel, so the solve runs on float32 copies of the
                          bf16 keys and values and X is cast back to bf16 for SDPA,
                          which is how the reference's path can run on bf16 tensors.
  Triton op (config 3)    parallel_lucid_path_attention (lucid_path/triton_code/
                          parallel.py:180-241) with flash-linear-attention's helper
                          kernels, bf16, forward and backward.

Each function raises RuntimeError("unavailable: ...") when the copy is missing.
"""
from __future__ import annotations

import importlib.util
import os
import sys
import types
import typing

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")


def available() -> bool:
    return os.path.exists(os.path.join(REF, "modeling_lucid.py"))


def load_modeling_lucid():
    """modeling_lucid.py as the module transformers.models.llama.modeling_lucid (its
    imports expect that package), with the one name transformers 5.x dropped."""
    path = os.path.join(REF, "modeling_lucid.py")
    if not os.path.exists(path):
        raise RuntimeError("unavailable: baseline/_ref/modeling_lucid.py missing (run baseline/install_ref.py)")
    name = "transformers.models.llama.modeling_lucid"
    if name in sys.modules:
        return sys.modules[name]
    import transformers.utils
    if not hasattr(transformers.utils, "LossKwargs"):
        class LossKwargs(typing.TypedDict, total=False):
            pass
        transformers.utils.LossKwargs = LossKwargs
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_path_op():
    """parallel_lucid_path_attention, its kernels imported as fla.ops.lucid_path (the
    flash-linear-attention fork the reference was written for)."""
    tc = os.path.join(REF, "lucid_path", "triton_code")
    if not os.path.exists(os.path.join(tc, "parallel.py")):
        raise RuntimeError("unavailable: baseline/_ref/lucid_path/triton_code missing (run baseline/install_ref.py)")
    import fla.ops  # noqa: F401
    if "fla.ops.lucid_path" not in sys.modules:
        pkg = types.ModuleType("fla.ops.lucid_path")
        pkg.__path__ = [tc]
        sys.modules["fla.ops.lucid_path"] = pkg
    from fla.ops.lucid_path.parallel import parallel_lucid_path_attention
    return parallel_lucid_path_attention


def cuda_ms(torch, fn, steps: int, warmup: int) -> float:
    """Mean device time of fn() over `steps` calls after `warmup` calls (CUDA events on
    the current stream)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def torch_path_step(torch, mod, q, k, v, do, eps: float = 1e-5):
    """One training step of the reference's LUCID layer on the GPU.  q [B,Hq,N,D],
    k, v [B,Hkv,N,D], do [B,N,Hq,D] (bf16).  Returns (o, dq, dk, dv)."""
    from transformers import LlamaConfig
    B, Hq, N, D = q.shape
    Hkv = k.shape[1]
    key = (B, Hq, Hkv, D, str(q.device))
    att = _ATT.get(key)
    if att is None:
        cfg = LlamaConfig(hidden_size=Hq * D, num_attention_heads=Hq, num_key_value_heads=Hkv, head_dim=D,
                          rms_norm_eps=eps, attention_bias=False)
        cfg.use_rope = False
        att = mod.LucidAttention(cfg, 0).to(q.device)
        att.train()
        _ATT.clear()
        _ATT[key] = att
    qq, kk, vv = (t.detach().requires_grad_(True) for t in (q, k, v))
    mask = att.create_causal_mask(qq, kk, 0)
    x = att.get_v_prime(kk.float(), vv.float(), att.scaling, mask).to(torch.bfloat16)
    o, _ = att.eager_lucid_attention_forward(qq, kk, x, att.scaling, mask)
    o.backward(do)
    return o.detach(), qq.grad, kk.grad, vv.grad


_ATT: dict = {}


def _max_abs(torch, a, b) -> float:
    return float((a.double() - b.double()).abs().max())


def torch_path_cfg2(torch, q, k, v, do, ours, steps: int = 3, warmup: int = 1, heads: int = 8):
    """Time the reference torch path at our config, and measure both its and our
    deviation from the float32 reference (oracle/torch_blockwise.py) on batch 0,
    heads [0, heads).  ours = (o, dq, dk, dv) of our op on the same inputs."""
    mod = load_modeling_lucid()
    ms = cuda_ms(torch, lambda: torch_path_step(torch, mod, q, k, v, do), steps, warmup)
    ref_out = torch_path_step(torch, mod, q, k, v, do)
    torch.cuda.synchronize()
    from oracle import torch_blockwise as tb
    hs = slice(0, heads)
    f = lambda t: t[0, hs].float()
    r = tb.lucid_fwd_bwd(f(q), f(k), f(v), do[0, :, hs].transpose(0, 1).float())
    names = ("o", "dq", "dk", "dv")
    pick = (lambda t: t[0, :, hs].transpose(0, 1), lambda t: t[0, hs], lambda t: t[0, hs], lambda t: t[0, hs])
    dev_ref = {n: _max_abs(torch, p(t), r[n]) for n, p, t in zip(names, pick, ref_out)}
    dev_ours = {n: _max_abs(torch, p(t), r[n]) for n, p, t in zip(names, pick, ours)}
    del r, ref_out
    torch.cuda.empty_cache()
    return {
        "impl": "reference torch path (modeling_lucid.py get_v_prime with a float32 solve + SDPA bf16, autograd)",
        "ms_per_step": ms,
        "max_abs_vs_fp32": dev_ref,
        "ours_max_abs_vs_fp32": dev_ours,
        "ours_over_reference_deviation": {n: dev_ours[n] / max(dev_ref[n], 1e-30) for n in names},
        "compared_on": f"batch 0, heads 0-{heads - 1}, float32 reference oracle/torch_blockwise.py",
    }


def triton_path(torch, k, v, w, beta, do, ours=None, steps: int = 3, warmup: int = 2, check: bool = True):
    """Time the reference Triton op (bf16) on [B,T,H,K] inputs, and measure its and
    our deviation from the float64 block restatement (oracle/path_oracle.py) on
    (batch 0, head 0).  ours = (o, dk, dv, dw, dbeta) of our op on the same inputs."""
    op = load_path_op()
    leaves = [t.detach().requires_grad_(True) for t in (k, v, w, beta)]

    def step():
        for t in leaves:
            t.grad = None
        o, _ = op(*leaves)
        o.backward(do)
        return o

    ms = cuda_ms(torch, step, steps, warmup)
    out = {"impl": "reference Triton op parallel_lucid_path_attention (lucid_path/triton_code) + fla helpers, bf16",
           "ms_per_step": ms}
    if not check:
        return out
    o = step().detach()
    torch.cuda.synchronize()
    got = (o, leaves[0].grad, leaves[1].grad, leaves[2].grad, leaves[3].grad)
    import numpy as np
    from oracle.path_oracle import path_bwd_blockwise, path_fwd_blockwise
    sl = lambda t: t[0:1, :, 0:1].detach().double().cpu().numpy()
    kk, vv, ww, dd = sl(k), sl(v), sl(w), sl(do)
    bb = beta[0:1, :, 0:1].detach().double().cpu().numpy()
    o_ref, _ = path_fwd_blockwise(kk, vv, ww, bb)
    _, dk_ref, dv_ref, dw_ref, db_ref = path_bwd_blockwise(kk, vv, ww, bb, dd)
    refs = (o_ref, dk_ref, dv_ref, dw_ref, db_ref)
    names = ("o", "dk", "dv", "dw", "dbeta")
    pick = lambda t: t[0:1, :, 0:1].detach().double().cpu().numpy()
    out["max_abs_vs_fp64"] = {n: float(np.abs(pick(t) - r).max()) for n, t, r in zip(names, got, refs)}
    if ours is not None:
        out["ours_max_abs_vs_fp64"] = {n: float(np.abs(pick(t) - r).max()) for n, t, r in zip(names, ours, refs)}
        out["ours_over_reference_deviation"] = {
            n: out["ours_max_abs_vs_fp64"][n] / max(out["max_abs_vs_fp64"][n], 1e-30) for n in names}
    out["compared_on"] = "batch 0, head 0, float64 block restatement oracle/path_oracle.py"
    return out
