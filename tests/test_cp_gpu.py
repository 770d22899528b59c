"""Context-parallel LUCID attention (lucid_b200/cp.py) on the B200 kernels.

* loopback (one GPU), contiguous chunks: W ranks run one after another in
  one process, the forward in rank order and the backward in reverse rank
  order, their messages passed through an in-process mailbox.  Every
  dependency of the chain points from an earlier-run rank to a later-run one,
  and the kernels never wait on another launch, so this runs the
  partial-range kernels and the whole protocol without a second GPU.
* loopback (one GPU), zigzag: every rank owns an early and a late segment, so
  the ranks' steps interleave; each rank runs in its own host thread, all on
  the same CUDA stream (GPU work executes in host order, one kernel at a
  time), a receive blocking its thread (bounded) until the sender has
  enqueued the message's copy.
* two GPUs over NCCL, contiguous and zigzag (skipped with fewer GPUs).
The gathered output and gradients must match the float64 oracle like the
single-GPU op does, and the single-GPU op itself closely (same kernels, same
accumulation order)."""
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


def _grad_out():
    import torch
    g = torch.Generator().manual_seed(18)
    B, Hq, N, D = (CASE[k] for k in ("B", "Hq", "N", "D"))
    return torch.randn(B, N, Hq, D, generator=g).bfloat16()


def _check_against_oracle(o, dq, dk, dv):
    from oracle.lucid_oracle import lucid_fwd_bwd
    q, k, v = (t.double().numpy() for t in _inputs())
    ro, rdq, rdk, rdv = lucid_fwd_bwd(q, k, v, _grad_out().double().numpy(), CASE["D"] ** -0.5, 1e-5)
    for nm, got, ref in (("o", o, ro), ("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv)):
        assert np.all(np.isfinite(got)), nm
        err = np.abs(got - ref) - (1e-2 + 2.0 ** -8 * np.abs(ref))
        assert err.max() <= 0, f"{nm}: max err {np.abs(got - ref).max():.3e}"


class _Req:
    def __init__(self, fn=None):
        self.fn = fn

    def wait(self):
        if self.fn:
            self.fn()


def _single_gpu(dev):
    import torch
    from lucid_b200.ops import lucid_attention
    q, k, v = _inputs()
    qs, ks, vs = (t.to(dev).requires_grad_() for t in (q, k, v))
    o = lucid_attention(qs, ks, vs)
    o.backward(_grad_out().to(dev))
    torch.cuda.synchronize()
    return [t.detach().float().cpu().numpy() for t in (o, qs.grad, ks.grad, vs.grad)]


def _close_to_single_gpu(got, ref):
    for nm, g, r in zip(("o", "dq", "dk", "dv"), got, ref):
        assert np.abs(g - r).max() <= 2.0 ** -7 * np.abs(r).max(), (nm, float(np.abs(g - r).max()))


def test_cp_loopback_fwd_bwd_matches_oracle_and_single_gpu(cuda_device):
    """Three ranks with unequal chunks (train_bounds) and two head groups."""
    import torch
    from lucid_b200.cp import ChunkProtocol, KernelBackend, Layout, train_bounds
    q, k, v = _inputs()
    do = _grad_out()
    B, Hq, H, N, D = (CASE[x] for x in ("B", "Hq", "H", "N", "D"))
    W = 3
    bounds = train_bounds(N, W)
    assert len(set(bounds[r + 1] - bounds[r] for r in range(W))) > 1
    layout = Layout.contiguous(bounds)
    mail = {}
    protos = []
    for r in range(W):
        be = KernelBackend(B, H, Hq, layout, D, D ** -0.5, 1e-5, r, W, CASE["groups"], cuda_device)
        pr = ChunkProtocol.__new__(ChunkProtocol)
        pr.be, pr.group, pr.rank, pr.world = be, None, r, W

        def send(t, j, r=r):
            mail.setdefault((r, j), []).append(t.clone())
            return _Req()

        def recv(t, j, r=r):
            box = mail[(j, r)]   # the sender ran first, so its message is queued
            return _Req(lambda: t.copy_(box.pop(0)))
        pr._send, pr._recv = send, recv
        protos.append(pr)
    dev = cuda_device
    outs = {}
    for r in range(W):
        rows = slice(bounds[r], bounds[r + 1])
        outs[r] = protos[r].run(q[:, :, rows].to(dev), k[:, :, rows].to(dev), v[:, :, rows].to(dev))
    grads = {}
    for r in reversed(range(W)):
        rows = slice(bounds[r], bounds[r + 1])
        grads[r] = protos[r].backward(do[:, rows].to(dev))
    torch.cuda.synchronize()
    assert not any(mail.values()), "unconsumed messages"
    o = torch.cat([outs[r] for r in range(W)], 1).float().cpu().numpy()
    dq, dk, dv = (torch.cat([grads[r][i] for r in range(W)], 2).float().cpu().numpy() for i in range(3))
    _check_against_oracle(o, dq, dk, dv)
    # the single-GPU op: same kernels, same accumulation order per block
    _close_to_single_gpu((o, dq, dk, dv), _single_gpu(dev))


def _local_index(layout, rank):
    import torch
    return torch.cat([torch.arange(layout.lo(s), layout.hi(s)) for s in layout.mine(rank)])


def _reassemble(parts, layout, axis):
    shape = list(parts[0].shape)
    shape[axis] = layout.N
    out = np.zeros(shape, dtype=parts[0].dtype)
    for r, part in enumerate(parts):
        idx = [slice(None)] * len(shape)
        idx[axis] = _local_index(layout, r).numpy()
        out[tuple(idx)] = part
    return out


@pytest.mark.parametrize("W", [2, 3])
def test_cp_zigzag_threaded_loopback_matches_oracle_and_single_gpu(cuda_device, W):
    """Zigzag layout: every rank owns segments r and 2W-1-r (two segments per rank:
    local row offsets, dV kept across segments, interleaved ranks)."""
    import threading
    import torch
    from lucid_b200.cp import ChunkProtocol, KernelBackend, zigzag_layout
    q, k, v = _inputs()
    do = _grad_out()
    B, Hq, H, N, D = (CASE[x] for x in ("B", "Hq", "H", "N", "D"))
    layout = zigzag_layout(N, W)
    assert all(len(layout.mine(r)) == 2 for r in range(W))
    dev = cuda_device
    lock = threading.Lock()
    mail, events = {}, {}

    def box(src, dst, n):
        with lock:
            key = (src, dst, n)
            if key not in events:
                events[key] = threading.Event()
            return key, events[key]

    class Req:
        def __init__(self, fn=None):
            self.fn = fn

        def wait(self):
            if self.fn:
                self.fn()

    results, errors = {}, {}

    def rank_main(r):
        try:
            torch.cuda.set_device(dev)
            be = KernelBackend(B, H, Hq, layout, D, D ** -0.5, 1e-5, r, W, CASE["groups"], dev)
            pr = ChunkProtocol.__new__(ChunkProtocol)
            pr.be, pr.group, pr.rank, pr.world = be, None, r, W
            sent, recvd = {}, {}

            def send(t, j):
                n = sent[j] = sent.get(j, -1) + 1
                key, ev = box(r, j, n)
                mail[key] = t.clone()   # enqueued on the shared stream after t's producer
                ev.set()
                return Req()

            def recv(t, j):
                n = recvd[j] = recvd.get(j, -1) + 1
                key, ev = box(j, r, n)

                def fn():
                    if not ev.wait(timeout=120):
                        raise TimeoutError(f"rank {r}: message {n} from rank {j} never came")
                    src = mail.pop(key)
                    assert src.shape == t.shape, (src.shape, t.shape)
                    t.copy_(src)
                return Req(fn)
            pr._send, pr._recv = send, recv
            idx = _local_index(layout, r)
            o = pr.run(q[:, :, idx].to(dev), k[:, :, idx].to(dev), v[:, :, idx].to(dev))
            g = pr.backward(do[:, idx].to(dev))
            torch.cuda.synchronize()
            results[r] = [t.float().cpu().numpy() for t in (o,) + tuple(g)]
        except Exception as e:  # noqa: BLE001
            errors[r] = e

    threads = [threading.Thread(target=rank_main, args=(r,)) for r in range(W)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=600)
    assert not errors, errors
    assert len(results) == W
    o = _reassemble([results[r][0] for r in range(W)], layout, 1)
    dq, dk, dv = (_reassemble([results[r][i] for r in range(W)], layout, 2) for i in (1, 2, 3))
    _check_against_oracle(o, dq, dk, dv)
    _close_to_single_gpu((o, dq, dk, dv), _single_gpu(dev))


def _worker(rank, world, port, out_dir, mode="contiguous"):
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
        from lucid_b200.cp import Layout, cp_lucid_attention, even_bounds, zigzag_layout
        q, k, v = _inputs()
        N = CASE["N"]
        layout = zigzag_layout(N, world) if mode == "zigzag" else Layout.contiguous(even_bounds(N, world))
        rows = _local_index(layout, rank)
        qs, ks, vs = (t[:, :, rows].to(dev).requires_grad_() for t in (q, k, v))
        o = cp_lucid_attention(qs, ks, vs, head_groups=CASE["groups"], layout=layout)
        o.backward(_grad_out()[:, rows].to(dev))
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f"o{rank}.npy"), o.detach().float().cpu().numpy())
        for nm, t in (("dq", qs), ("dk", ks), ("dv", vs)):
            np.save(os.path.join(out_dir, f"{nm}{rank}.npy"), t.grad.float().cpu().numpy())
    except Exception as e:  # noqa: BLE001
        with open(os.path.join(out_dir, f"err{rank}.txt"), "w") as f:
            f.write(repr(e))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["contiguous", "zigzag"])
def test_cp_fwd_bwd_two_gpus_matches_oracle(tmp_path, mode):
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    from lucid_b200.cp import Layout, even_bounds, zigzag_layout
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), mode), nprocs=world, start_method="spawn")
    for r in range(world):
        assert not (tmp_path / f"err{r}.txt").exists(), (tmp_path / f"err{r}.txt").read_text()
    N = CASE["N"]
    layout = zigzag_layout(N, world) if mode == "zigzag" else Layout.contiguous(even_bounds(N, world))
    o = _reassemble([np.load(tmp_path / f"o{r}.npy") for r in range(world)], layout, 1)
    dq, dk, dv = (_reassemble([np.load(tmp_path / f"{nm}{r}.npy") for r in range(world)], layout, 2)
                  for nm in ("dq", "dk", "dv"))
    _check_against_oracle(o, dq, dk, dv)
