"""Context-parallel LUCID forward (lucid_b200/cp.py) on real GPUs over NCCL:
two ranks each own half of the sequence; the gathered output must match the
float64 oracle like the single-GPU op does.  Needs at least two GPUs (skipped
otherwise)."""
import os
import socket

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

CASE = dict(B=1, Hq=4, H=2, N=4096, D=128, groups=2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    import torch
    g = torch.Generator().manual_seed(17)
    B, Hq, H, N, D = (CASE[k] for k in ("B", "Hq", "H", "N", "D"))
    q = (torch.randn(B, Hq, N, D, generator=g) * D ** -0.5).bfloat16()
    k = (0.6 * torch.randn(B, H, 1, D, generator=g) + 0.8 * torch.randn(B, H, N, D, generator=g)).bfloat16()
    v = torch.randn(B, H, N, D, generator=g).bfloat16()
    return q, k, v


def _worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        from lucid_b200.cp import cp_lucid_attention_forward
        q, k, v = _inputs()
        C = CASE["N"] // world
        rows = slice(rank * C, (rank + 1) * C)
        o = cp_lucid_attention_forward(q[:, :, rows].to(dev), k[:, :, rows].to(dev), v[:, :, rows].to(dev),
                                       head_groups=CASE["groups"])
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f"o{rank}.npy"), o.float().cpu().numpy())
    except Exception as e:  # noqa: BLE001
        with open(os.path.join(out_dir, f"err{rank}.txt"), "w") as f:
            f.write(repr(e))
    finally:
        dist.destroy_process_group()


def test_cp_forward_two_gpus_matches_oracle(tmp_path):
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    from oracle.lucid_oracle import lucid_fwd
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    for r in range(world):
        assert not (tmp_path / f"err{r}.txt").exists(), (tmp_path / f"err{r}.txt").read_text()
    o = np.concatenate([np.load(tmp_path / f"o{r}.npy") for r in range(world)], axis=1)
    q, k, v = (t.double().numpy() for t in _inputs())
    ref = lucid_fwd(q, k, v, CASE["D"] ** -0.5, 1e-5)[0]
    assert np.all(np.isfinite(o))
    err = np.abs(o - ref) - (1e-2 + 2.0 ** -8 * np.abs(ref))
    assert err.max() <= 0, np.abs(o - ref).max()
