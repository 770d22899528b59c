"""Generate the golden LUCID-Path fixtures from the reference implementation.

Runs the reference's own Triton op ``parallel_lucid_path_attention``
(lucid_path/triton_code/parallel.py:180-241 of saisuryadv/LUCID) in float32
under Triton's CPU interpreter (TRITON_INTERPRET=1), forward and backward,
and stores inputs (as bf16 bit patterns) and outputs (float32, including the
decode-time key cache of use_cache=True, prepare_k_cache.py) in ``path_*.npz``
next to this script.

The op imports its kernels as the package ``fla.ops.lucid_path`` (the
flash-linear-attention fork it was written for); this script registers the
reference directory under that name and applies the three shims the CPU
interpreter needs:
  * ``torch.cpu.device`` as a null context (fla's ``input_guard``);
  * a constant ``Autotuner._bench`` (no GPU to time fla's autotuned kernels);
  * the package alias above.
bf16 is not usable in the interpreter (it returns NaN), so the reference is
run in float32 on bf16-representable inputs.

It also stores ``pathattn_*.npz``: the PaTH softmax attention forward of the
same directory (intra_chunk_preprocess_fwd.py + parallel_path_fwd.py), o and the
log2-sum-exp L.

The reference checkout is only needed to regenerate; the fixtures are committed.

Usage:  python tests/golden/make_path_golden.py /path/to/LUCID
"""
from __future__ import annotations

import contextlib
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

CASES = {
    # name: (seed, B, T, H, K, HQ, explicit q)
    "path_t256_k128": (1, 1, 256, 1, 128, 1, False),
    "path_gqa_t200_k128": (2, 1, 200, 1, 128, 2, True),
    "path_t320_k32": (3, 1, 320, 2, 32, 2, False),
}


def load_reference(root: str):
    os.environ["TRITON_INTERPRET"] = "1"
    import torch
    torch.cpu.device = lambda i=None: contextlib.nullcontext()
    import triton.runtime.autotuner as at
    at.Autotuner._bench = lambda *a, **k: [1.0, 1.0, 1.0]
    import fla.ops  # noqa: F401
    pkg = types.ModuleType("fla.ops.lucid_path")
    pkg.__path__ = [os.path.join(root, "lucid_path", "triton_code")]
    sys.modules["fla.ops.lucid_path"] = pkg
    from fla.ops.lucid_path.parallel import parallel_lucid_path_attention
    return parallel_lucid_path_attention


ATTN_CASES = {
    # name: (seed, B, T, H, K, HQ, explicit q)
    "pathattn_t256_k128": (4, 1, 256, 1, 128, 1, False),
    "pathattn_gqa_t200_k128": (5, 1, 200, 1, 128, 2, True),
}


def reference_path_attention(root: str, q, k, v, w, beta, scale):
    """The PaTH softmax attention forward as the reference's kernels compute it:
    T_inv (parallel.py:40-51), intra_chunk_preprocess_fwd_fn (diagonal blocks,
    q_new / k_new / w2) then parallel_path_fwd_fn (off-diagonal blocks, online
    softmax).  The reference ships these two kernels without a caller; this is the
    composition their interfaces imply, with BT = BS = 64."""
    import torch
    from fla.ops.common.chunk_scaled_dot_kkt import chunk_scaled_dot_kkt_fwd
    from fla.ops.utils.solve_tril import solve_tril
    from fla.ops.lucid_path.intra_chunk_preprocess_fwd import intra_chunk_preprocess_fwd_fn
    from fla.ops.lucid_path.parallel_path_fwd import parallel_path_fwd_fn
    A = chunk_scaled_dot_kkt_fwd(k=w, beta=beta, cu_seqlens=None, chunk_size=64, output_dtype=torch.float32)
    A = solve_tril(A=A, cu_seqlens=None, output_dtype=w.dtype)
    q_new, k_new, w2, o, L, M = intra_chunk_preprocess_fwd_fn(q, k, v, w, beta, None, A, scale, 64, None)
    o, L = parallel_path_fwd_fn(q_new, k_new, v, o, None, w, w2, scale, L, M, None, 64, 64)
    return o, L


def bf16_bits(a: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(a, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def main(root: str):
    import torch
    from oracle.path_oracle import make_path_inputs
    op = load_reference(root)
    for name, (seed, B, T, H, K, HQ, with_q) in CASES.items():
        d = make_path_inputs(seed, B, T, H, K, HQ, with_q)
        t = {n: (torch.tensor(d[n], dtype=torch.float32, requires_grad=n != "do") if d[n] is not None else None)
             for n in d}
        o, kc = op(t["k"], t["v"], t["w"], t["beta"], q=t["q"], use_cache=True)
        o.backward(t["do"])
        out = dict(o=o.detach().numpy(), dk=t["k"].grad.numpy(), dv=t["v"].grad.numpy(),
                   dw=t["w"].grad.numpy(), dbeta=t["beta"].grad.numpy(), k_cache=kc.detach().numpy())
        if with_q:
            out["dq"] = t["q"].grad.numpy()
        arrs = {f"{n}_bf16": bf16_bits(d[n]) for n in ("q", "k", "v", "w", "beta", "do") if d[n] is not None}
        arrs.update({n: a.astype(np.float32) for n, a in out.items()})
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrs)
        print(name, {n: float(np.abs(a).max()) for n, a in out.items()})
    for name, (seed, B, T, H, K, HQ, with_q) in ATTN_CASES.items():
        d = make_path_inputs(seed, B, T, H, K, HQ, with_q)
        t = {n: (torch.tensor(d[n], dtype=torch.float32) if d[n] is not None else None) for n in d}
        q = t["q"] if with_q else t["k"]
        o, L = reference_path_attention(root, q, t["k"], t["v"], t["w"], t["beta"], K ** -0.5)
        arrs = {f"{n}_bf16": bf16_bits(d[n]) for n in ("q", "k", "v", "w", "beta") if d[n] is not None}
        arrs.update(o=o.numpy().astype(np.float32), lse=L.numpy().astype(np.float32))
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrs)
        print(name, float(np.abs(o.numpy()).max()), float(np.abs(L.numpy()).max()))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "LUCID")
