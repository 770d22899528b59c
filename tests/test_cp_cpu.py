"""The context-parallel chunk protocol (lucid_b200/cp.py) on CPU gloo ranks.

Each rank runs ChunkProtocol with the float64 CPU backend; the gathered
outputs must equal the single-process oracle on the whole sequence.  Failure
handling: a rank that dies before sending makes its successor's receive fail
with an error instead of hanging."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT

SEQ = dict(B=1, Hq=4, H=2, N=384, D=16)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    g = torch.Generator().manual_seed(5)
    B, Hq, H, N, D = (SEQ[k] for k in ("B", "Hq", "H", "N", "D"))
    q = torch.randn(B, Hq, N, D, generator=g, dtype=torch.float64)
    k = 0.6 * torch.randn(B, H, 1, D, generator=g, dtype=torch.float64) + 0.8 * torch.randn(B, H, N, D, generator=g,
                                                                                            dtype=torch.float64)
    v = torch.randn(B, H, N, D, generator=g, dtype=torch.float64)
    return q, k, v


def _grad_out():
    g = torch.Generator().manual_seed(6)
    B, Hq, N, D = (SEQ[k] for k in ("B", "Hq", "N", "D"))
    return torch.randn(B, N, Hq, D, generator=g, dtype=torch.float64)


def _layout(world, mode):
    from lucid_b200.cp import Layout, balanced_bounds, even_bounds, train_bounds, zigzag_layout
    N = SEQ["N"]
    if mode == "zigzag":
        return zigzag_layout(N, world, align=32)
    if mode == "train":
        return Layout.contiguous(train_bounds(N, world, align=64))
    if mode == "balanced":
        return Layout.contiguous(balanced_bounds(N, world, align=64))
    return Layout.contiguous(even_bounds(N, world))


def _local_index(layout, rank):
    """The global rows a rank holds, in its local order (its segments in sequence order)."""
    return torch.cat([torch.arange(layout.lo(s), layout.hi(s)) for s in layout.mine(rank)])


def _worker(rank, world, port, groups, mode, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from datetime import timedelta
    from cp_cpu_backend import CpuBackend
    from lucid_b200.cp import ChunkProtocol
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    q, k, v = _inputs()
    layout = _layout(world, mode if not mode.startswith("die") else "even")
    rows = _local_index(layout, rank)
    be = CpuBackend(SEQ["B"], SEQ["H"], SEQ["Hq"], layout, SEQ["D"], SEQ["D"] ** -0.5, 1e-5, rank, world, groups)
    try:
        if mode == "die" and rank == 0:
            os._exit(0)   # leaves without sending anything
        proto = ChunkProtocol(be)
        o = proto.run(q[:, :, rows], k[:, :, rows], v[:, :, rows])
        np.save(os.path.join(out_dir, f"o{rank}.npy"), o.numpy())
        if mode == "die_bwd" and rank == world - 1:
            os._exit(0)   # finishes the forward, then leaves without sending its backward inputs
        dq, dk, dv = proto.backward(_grad_out()[:, rows])
        for nm, t in (("dq", dq), ("dk", dk), ("dv", dv)):
            np.save(os.path.join(out_dir, f"{nm}{rank}.npy"), t.numpy())
    except Exception as e:  # noqa: BLE001 - the failure test inspects it
        with open(os.path.join(out_dir, f"err{rank}.txt"), "w") as f:
            f.write(repr(e))
    finally:
        if not mode.startswith("die"):
            dist.destroy_process_group()


def _gather(tmp_path, name, world, layout, axis):
    """Reassemble the per-rank local outputs into sequence order."""
    parts = [np.load(tmp_path / f"{name}{r}.npy") for r in range(world)]
    shape = list(parts[0].shape)
    shape[axis] = layout.N
    out = np.zeros(shape, dtype=parts[0].dtype)
    for r in range(world):
        idx = [slice(None)] * len(shape)
        idx[axis] = _local_index(layout, r).numpy()
        out[tuple(idx)] = parts[r]
    return out


@pytest.mark.parametrize("world,groups,mode", [(2, 1, "even"), (3, 2, "even"), (3, 2, "balanced"),
                                               (4, 2, "train"), (2, 2, "zigzag"), (3, 2, "zigzag"),
                                               (4, 1, "zigzag")])
def test_cp_protocol_matches_oracle(tmp_path, world, groups, mode):
    """Forward and backward chains on gloo ranks: the gathered O, dQ, dK, dV equal
    the float64 oracle on the whole sequence (contiguous chunks and the zigzag,
    where every rank owns an early and a late segment)."""
    from oracle.lucid_oracle import lucid_bwd, lucid_fwd
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, groups, mode, str(tmp_path)), nprocs=world, start_method="spawn")
    for r in range(world):
        assert not (tmp_path / f"err{r}.txt").exists(), (tmp_path / f"err{r}.txt").read_text()
    layout = _layout(world, mode)
    o = _gather(tmp_path, "o", world, layout, 1)
    q, k, v = (t.numpy() for t in _inputs())
    ref = lucid_fwd(q, k, v, SEQ["D"] ** -0.5, 1e-5)[0]
    np.testing.assert_allclose(o, ref, rtol=1e-10, atol=1e-10)
    dq, dk, dv = lucid_bwd(q, k, v, _grad_out().numpy(), SEQ["D"] ** -0.5, 1e-5)
    for nm, r_ in (("dq", dq), ("dk", dk), ("dv", dv)):
        got = _gather(tmp_path, nm, world, layout, 2)
        np.testing.assert_allclose(got, r_, rtol=1e-9, atol=1e-9, err_msg=nm)


@pytest.mark.parametrize("mode,dead,waiting", [("die", 0, 1), ("die_bwd", 1, 0)])
def test_cp_protocol_reports_a_dead_peer(tmp_path, mode, dead, waiting):
    """A rank that leaves (before the forward's keys, or after the forward but
    before the backward's messages) makes its peer's next receive end with an
    error (the process group timeout is 10 s) instead of hanging."""
    port = _free_port()
    ctx = mp.start_processes(_worker, args=(2, port, 1, mode, str(tmp_path)), nprocs=2, start_method="spawn",
                             join=False)
    import time
    deadline = time.time() + 120
    while any(p.is_alive() for p in ctx.processes) and time.time() < deadline:
        time.sleep(0.5)
    hung = [p for p in ctx.processes if p.is_alive()]
    for p in hung:
        p.kill()
    assert not hung, "a rank hung after its peer died"
    assert (tmp_path / f"err{waiting}.txt").exists()


def test_zigzag_balances_forward_and_backward_work():
    """Per-rank forward work (rows t cost ~t) and backward column work (~N - t)
    are both equal for the zigzag; contiguous chunks can balance only one."""
    from lucid_b200.cp import Layout, balanced_bounds, zigzag_layout
    N, W = 131072, 8

    def work(L, f):
        return [sum(f(L.hi(s)) - f(L.lo(s)) for s in L.mine(r)) for r in range(W)]
    fwd = lambda x: x * x / 2            # integral of t
    col = lambda x: N * x - x * x / 2    # integral of N - t
    z = zigzag_layout(N, W)
    for f in (fwd, col):
        w = work(z, f)
        assert max(w) / min(w) < 1.001
    c = Layout.contiguous(balanced_bounds(N, W))
    assert max(work(c, fwd)) / min(work(c, fwd)) < 1.05
    assert max(work(c, col)) / min(work(c, col)) > 5


def test_balanced_bounds_equalise_causal_work():
    from lucid_b200.cp import balanced_bounds
    N, W = 131072, 8
    b = balanced_bounds(N, W)
    assert b[0] == 0 and b[-1] == N and all(x % 256 == 0 for x in b)
    work = [(b[r + 1] ** 2 - b[r] ** 2) / N ** 2 for r in range(W)]
    assert max(work) < 1.02 / W


class _Req:
    def wait(self):
        pass


class _NullBackend:
    """Computes nothing: every tensor is a tag naming the message it carries
    (kind, heads, segment), so that the simulation can check that both ends of
    a pair agree on every message."""

    def __init__(self, G, layout):
        self.G, self.H, self.Hg, self.layout = G, 2, 1, layout

    def set_local(self, q, k):
        pass

    def empty_chunk(self, heads, s):
        return ("chunk", heads, s)

    def keys(self, s):
        return ("chunk", self.H, s)

    def store_keys(self, s, buf):
        pass

    def prep(self):
        pass

    def store_values(self, g, s, buf):
        pass

    def solve(self, t, g, v):
        pass

    def own_values(self, t, g):
        return ("chunk", self.Hg, t)

    def attend(self, t, g):
        pass

    def finish(self):
        return None

    def set_grad(self, do):
        pass

    def empty_grad_inputs(self, s):
        return [("gin", 0, s), ("gin", 1, s)]

    def grad_inputs(self, s):
        return [("gin", 0, s), ("gin", 1, s)]

    def store_grad_inputs(self, s, bufs):
        pass

    def prep_later(self):
        pass

    def attn_col(self, t, g):
        pass

    def store_dv(self, g, s, buf):
        pass

    def solve_col(self, t, g):
        pass

    def own_dv(self, t, g):
        return ("chunk", self.Hg, t)

    def rows(self, t, g):
        pass

    def finish_grad(self):
        return None


def _schedule(rank, world, G, layout):
    """The point-to-point operations rank `rank` issues, in issue order, each
    with the tag of the message it carries."""
    from lucid_b200.cp import ChunkProtocol
    ops = []
    proto = ChunkProtocol.__new__(ChunkProtocol)
    proto.be, proto.group, proto.rank, proto.world = _NullBackend(G, layout), None, rank, world
    proto._send = lambda t, j: (ops.append(("send", j, t)), _Req())[1]
    proto._recv = lambda t, j: (ops.append(("recv", j, t)), _Req())[1]
    proto.run(None, None, None)
    proto.backward(None)
    return ops


@pytest.mark.parametrize("world", [2, 3, 4, 8])
@pytest.mark.parametrize("G", [1, 2, 8])
@pytest.mark.parametrize("layout", ["contiguous", "zigzag"])
def test_cp_schedule_cannot_deadlock_even_fully_serialised(world, G, layout):
    """Forward then backward chain.  Worst case for NCCL point-to-point: every
    rank runs all of its sends and receives strictly in issue order (one queue
    per rank, as a single eager communicator does).  A send and a receive
    complete together when each is at the head of its rank's queue and both
    carry the same message (kind, heads, segment); the whole schedule must
    drain.  Also checks, per pair and direction, that the two ends list the
    same messages in the same order (what NCCL's in-order matching needs even
    when the ranks are not serialised)."""
    from lucid_b200.cp import Layout, even_bounds, zigzag_layout
    N = 256 * 2 * world
    L = zigzag_layout(N, world) if layout == "zigzag" else Layout.contiguous(even_bounds(N, world))
    sched = [list(_schedule(r, world, G, L)) for r in range(world)]
    for a in range(world):
        for b in range(world):
            if a != b:
                sent = [t for op, j, t in sched[a] if op == "send" and j == b]
                got = [t for op, j, t in sched[b] if op == "recv" and j == a]
                assert sent == got, f"pair {a}->{b}: sends {sent} vs receives {got}"
    queues = [list(q) for q in sched]
    progress = True
    while progress and any(queues):
        progress = False
        for r in range(world):
            if not queues[r]:
                continue
            op, j, t = queues[r][0]
            if op == "send" and queues[j] and queues[j][0] == ("recv", r, t):
                queues[r].pop(0)
                queues[j].pop(0)
                progress = True
    assert not any(queues), f"deadlock: heads {[q[0] if q else None for q in queues]}"
