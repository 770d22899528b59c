"""LUCID-Path argument checks (CPU): the drop-in rejects what the reference op
rejects (lucid_path/triton_code/parallel.py:230-239 asserts), with an error that
callers of the reference catch as AssertionError, before any device work; valid
arguments on CPU tensors raise instead of falling back to a CPU path."""
import pytest
import torch

from lucid_b200.path import PathArgumentError, parallel_lucid_path_attention, parallel_path_attention_fwd


def _args(B=1, T=64, H=2, K=128, V=128, HQ=None):
    k = torch.zeros(B, T, H, K, dtype=torch.bfloat16)
    v = torch.zeros(B, T, H, V, dtype=torch.bfloat16)
    w = torch.zeros(B, T, H, K, dtype=torch.bfloat16)
    beta = torch.zeros(B, T, H, dtype=torch.bfloat16)
    q = None if HQ is None else torch.zeros(B, T, HQ, K, dtype=torch.bfloat16)
    return k, v, w, beta, q


@pytest.mark.parametrize("case", ["head_dim", "v_head_dim", "q_head_dim", "w_shape", "beta_heads", "g",
                                  "query_heads", "varlen_batch"])
def test_rejects_what_the_reference_asserts(case):
    k, v, w, beta, q = _args()
    kw = {}
    if case == "head_dim":
        k, v, w, beta, q = _args(K=48)
    elif case == "v_head_dim":
        k, v, w, beta, q = _args(V=96)
    elif case == "q_head_dim":
        q = torch.zeros(1, 64, 2, 64, dtype=torch.bfloat16)
    elif case == "w_shape":
        w = w[:, :32]
    elif case == "beta_heads":
        beta = torch.zeros(1, 64, 3, dtype=torch.bfloat16)
    elif case == "g":
        kw["g"] = torch.zeros(1, 64, 2)
    elif case == "query_heads":
        k, v, w, beta, q = _args(H=2, HQ=3)
    elif case == "varlen_batch":
        k, v, w, beta, q = _args(B=2)
        kw["cu_seqlens"] = torch.tensor([0, 32, 64])
    with pytest.raises(AssertionError):
        parallel_lucid_path_attention(k, v, w, beta, q=q, **kw)
    with pytest.raises(PathArgumentError):
        parallel_lucid_path_attention(k, v, w, beta, q=q, **kw)


def test_path_attention_rejects_head_dim():
    k, v, w, beta, _ = _args(K=80)
    with pytest.raises(AssertionError):
        parallel_path_attention_fwd(None, k, v, w, beta)


@pytest.mark.parametrize("K", [128, 64])
def test_cpu_tensors_raise_without_fallback(K):
    k, v, w, beta, _ = _args(K=K, V=K)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        parallel_lucid_path_attention(k, v, w, beta)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        parallel_path_attention_fwd(None, k, v, w, beta)


def test_path_memory_groups_split_by_kv_head():
    """Group selection of the bounded-memory LUCID-Path schedule (workspace sizes from
    the C ABI, no GPU needed): the whole batch when it fits, else the largest kv-head
    group that fits, and a clear error when one head does not."""
    pytest.importorskip("torch")
    from lucid_b200 import _lib
    from lucid_b200.path import path_memory_groups
    lib = _lib.load()
    per = lambda b, h: (lib.lucid_path_fwd_workspace_bytes(b, 1000, h, 2 * h, 128)
                        + lib.lucid_path_bwd_workspace_bytes(b, 1000, h, 2 * h, 128))
    assert path_memory_groups(2, 1000, 4, 8, None, budget=per(2, 4)) == [(0, 2, 0, 4)]
    assert path_memory_groups(2, 1000, 4, 8, None, budget=per(1, 2)) == [(0, 1, 0, 2), (0, 1, 2, 4),
                                                                         (1, 2, 0, 2), (1, 2, 2, 4)]
    assert len(path_memory_groups(2, 1000, 4, 8, None, budget=per(1, 1))) == 8
    with pytest.raises(_lib.LucidError):
        path_memory_groups(2, 1000, 4, 8, None, budget=per(1, 1) - 1)
