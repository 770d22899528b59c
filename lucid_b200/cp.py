"""Context-parallel LUCID attention forward for long sequences (the 128K
configuration): one process per GPU, each rank owning a contiguous chunk of
C = N / world tokens of every (batch, head).

The reference runs long sequences on one GPU (the blockwise solver of
modeling_lucid.py:285-312 under gradient checkpointing); this module spreads
one sequence over the GPUs of a node:

  X = P^-1 V is a forward substitution, so chunk r needs the solved values
  X_j and the keys K_j of every earlier chunk j < r:
    R_r = V_r - sum_{j<r} exp(s K^_r K^_j^T - 1/s) X_j ,  X_r = P_rr^-1 R_r
  and the attention of chunk r's queries needs K_j and X_j of every j <= r.

Protocol (all point-to-point NCCL send/recv, no collective):
  1. every rank sends its raw keys to every later rank (they are an input,
     so this starts at once); a receiver normalises them (k^ only);
  2. the kv heads are split into head groups; for each group g in order,
     rank r waits for X_j(g) of every j < r, marks those row blocks solved
     (the wavefront solve's per-block flags), solves its own row blocks,
     sends its X_r(g) to every later rank and runs the attention of its own
     queries for the group.  Rank r solves group g while rank r-1 already
     works on group g+1, so the serial chain across ranks is pipelined over
     the head groups.
  Kernels never wait on another launch: every dependency is a stream-ordered
  NCCL receive, and the persistent kernels leave `reserve_sms` SMs free so
  the NCCL kernels of the other groups run alongside.

Backward (ChunkProtocol.backward, after run): a rank computes every
gradient of its own rows.  Its column passes (attention dX / dK over its
own key blocks, the transposed solve dV = P^-T dX and the column part of
dK^) need the rows after its chunk, its row passes (dQ, the row part of
dK^) only the rows before it, which the forward already brought in.  So
the messages mirror the forward's, flowing from higher to lower ranks:
  1. every rank sends q, dO, its raw keys, lse and delta = rowsum(dO o O)
     of its rows to every earlier rank (inputs and forward outputs, so
     this starts at once);
  2. for each head group in order, rank r waits for dV_j(g) of every
     j > r, publishes those blocks, runs its transposed solve, sends its
     dV_r(g) to every earlier rank, then runs the attention column pass of
     group g+1 and the row passes of group g while rank r-1 solves.
The chain of the backward runs from the last rank to the first.

Chunks may differ in length.  balanced_bounds equalises the forward's work
(the solve and the attention of row t cost ~t); train_bounds equalises the
forward plus the backward, whose column passes cost ~N-t and row passes ~t.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib

__all__ = ["cp_lucid_attention_forward", "cp_lucid_attention", "ChunkProtocol", "KernelBackend", "balanced_bounds",
           "even_bounds", "train_bounds"]


def even_bounds(N: int, world: int):
    """Chunk boundaries of equal contiguous chunks."""
    return [r * (N // world) for r in range(world)] + [N]


def balanced_bounds(N: int, world: int, align: int = 256):
    """Contiguous chunks of equal causal work: row r's solve and attention cost
    grows with r, so the chunk of rank r ends near N sqrt((r+1)/world)
    (rounded to `align` rows, 256 = one pair of 128-row blocks)."""
    b = [0]
    for r in range(1, world):
        x = int(round(N * (r / world) ** 0.5 / align)) * align
        b.append(min(max(x, b[-1] + align), N - (world - r) * align))
    return b + [N]


def train_bounds(N: int, world: int, align: int = 256, col: float = 1.0, row: float = 1.2, flat: float = 0.05):
    """Contiguous chunks of equal forward + backward work.  Per row t of an N-row
    sequence the work is modelled as col (N - t) + row t + flat N: the backward's
    column passes (attention dX / dK, transposed solve) cost ~N - t, the forward
    and the backward's row passes ~t, the row statistics a constant.  The default
    weights are the measured stage times of the single-GPU kernels (column passes
    34 ms, forward + row passes 42 ms, prep 3.5 ms at N = 32768)."""
    def work(x):  # cumulative work of rows [0, x), in units of N^2
        u = x / N
        return col * (u - u * u / 2) + row * u * u / 2 + flat * u
    total = work(N)
    b = [0]
    for r in range(1, world):
        target = total * r / world
        lo, hi = 0.0, float(N)
        for _ in range(60):
            mid = (lo + hi) / 2
            lo, hi = (mid, hi) if work(mid) < target else (lo, mid)
        x = int(round(lo / align)) * align
        b.append(min(max(x, b[-1] + align), N - (world - r) * align))
    return b + [N]


_PAIR_GROUPS = {}


def _pair_groups(group):
    """One process group per pair of ranks (created once, by every rank in the
    same order), so that point-to-point traffic between different pairs never
    queues behind one another (a single communicator runs its send/recv ops
    in issue order)."""
    ranks = dist.get_process_group_ranks(group) if group is not None else list(range(dist.get_world_size()))
    key = tuple(ranks)
    if key not in _PAIR_GROUPS:
        _PAIR_GROUPS[key] = {(a, b): dist.new_group([ranks[a], ranks[b]])
                             for a in range(len(ranks)) for b in range(a + 1, len(ranks))}
    return _PAIR_GROUPS[key], ranks


class ChunkProtocol:
    """The message schedule of the forward chain, independent of how the
    chunks are computed (``backend``) and of the process group's device.

    Every message flows from a lower to a higher rank, each pair of ranks has
    its own communicator, and both ends of a pair exchange their messages in
    the same order (keys, then the values of head group 0, 1, ...).  Rank r
    posts the receives of group g only after its sends of group g-1, so even
    if all of a rank's operations ran in issue order every wait would be on a
    (group, rank) that comes earlier: the schedule cannot deadlock."""

    def __init__(self, backend, group=None):
        self.be = backend
        self.group = group
        # a single process without a process group is a world of one
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.pairs, self.ranks = _pair_groups(group) if self.world > 1 else ({}, [0])

    def _send(self, t, j):
        lo, hi = min(self.rank, j), max(self.rank, j)
        return dist.isend(t, dst=self.ranks[j], group=self.pairs[lo, hi])

    def _recv(self, t, j):
        lo, hi = min(self.rank, j), max(self.rank, j)
        return dist.irecv(t, src=self.ranks[j], group=self.pairs[lo, hi])

    def run(self, q, k, v):
        be, r, W = self.be, self.rank, self.world
        be.set_local(q, k)
        # 1. raw keys flow to every later rank
        kbuf = {j: be.empty_chunk(be.H, j) for j in range(r)}
        reqs = [self._recv(kbuf[j], j) for j in range(r)]
        ksend = be.own_keys()
        sends = [self._send(ksend, j) for j in range(r + 1, W)]
        for rq in reqs:
            rq.wait()
        for j in range(r):
            be.store_keys(j, kbuf[j])
        be.prep()
        # 2. solved values, pipelined over head groups
        for g in range(be.G):
            xbuf = {j: be.empty_chunk(be.Hg, j) for j in range(r)}
            reqs = [self._recv(xbuf[j], j) for j in range(r)]
            for j in range(r):
                reqs[j].wait()
                be.store_values(g, j, xbuf[j])
            be.solve(g, v)
            xs = be.own_values(g)
            sends += [self._send(xs, j) for j in range(r + 1, W)]
            be.attend(g)
        for s in sends:
            s.wait()
        return be.finish()

    def backward(self, do):
        """Gradients of this rank's rows after run(): returns what the
        backend's finish_grad returns (dq, dk, dv of the chunk)."""
        be, r, W = self.be, self.rank, self.world
        be.set_grad(do)
        # 1. q, dO, raw keys, lse and delta flow to every earlier rank; receives
        #    from later ranks are posted latest-rank first and sends go to the
        #    nearest earlier rank first (the forward's order under r -> W-1-r)
        later = list(range(W - 1, r, -1))
        earlier = list(range(r - 1, -1, -1))
        bufs = {j: be.empty_grad_inputs(j) for j in later}
        reqs = {j: [self._recv(t, j) for t in bufs[j]] for j in later}
        mine = be.own_grad_inputs()
        sends = [self._send(t, j) for j in earlier for t in mine]
        for j in later:
            for rq in reqs[j]:
                rq.wait()
            be.store_grad_inputs(j, bufs[j])
        be.prep_later()
        # 2. dV flows to earlier ranks, pipelined over head groups
        be.attn_col(0)
        for g in range(be.G):
            dbuf = {j: be.empty_chunk(be.Hg, j) for j in later}
            reqs = [self._recv(dbuf[j], j) for j in later]
            for j, rq in zip(later, reqs):
                rq.wait()
                be.store_dv(g, j, dbuf[j])
            be.solve_col(g)
            dvs = be.own_dv(g)
            sends += [self._send(dvs, j) for j in earlier]
            if g + 1 < be.G:
                be.attn_col(g + 1)
            be.rows(g)
        for s in sends:
            s.wait()
        return be.finish_grad()


class KernelBackend:
    """The chunk computations on the B200 kernels (C ABI lucid_cp_*)."""

    def __init__(self, B, H, Hq, bounds, D, scale, eps, rank, world, head_groups, device, reserve_sms=8):
        if D != 128:
            raise NotImplementedError("head_dim must be 128")
        N = bounds[-1]
        if len(bounds) != world + 1 or bounds[0] != 0 or any(x % 256 for x in bounds[:-1]) or \
                any(bounds[j + 1] <= bounds[j] for j in range(world)) or N % 128:
            raise ValueError("chunk bounds must start at 0, increase, and sit on multiples of 256 rows")
        if H % head_groups or Hq % H:
            raise ValueError("head_groups must divide the kv heads and Hq must be a multiple of H")
        self.lib = _lib.load()
        self.B, self.H, self.Hq, self.N, self.D = B, H, Hq, N, D
        self.s, self.eps = float(scale), float(eps)
        self.r, self.W = rank, world
        self.G, self.Hg, self.Gq = head_groups, H // head_groups, Hq // H
        self.bounds = list(bounds)
        self.C = bounds[rank + 1] - bounds[rank]
        self.NB = N // 128
        self.blk_lo = bounds[rank] // 128
        self.blk_hi = bounds[rank + 1] // 128
        self.row0 = bounds[rank]
        self.dev = device
        n_sm = torch.cuda.get_device_properties(device).multi_processor_count
        self.max_ctas = max(1, n_sm - reserve_sms) if world > 1 else 0
        bf = dict(dtype=torch.bfloat16, device=device)
        self.Kf = torch.zeros(B, H, N, D, **bf)
        self.Qf = torch.zeros(B, Hq, N, D, **bf)
        self.khat = [torch.zeros(B, self.Hg, N, D, **bf) for _ in range(self.G)]
        self.x = [torch.zeros(B, self.Hg, N, D, **bf) for _ in range(self.G)]
        self.u = [torch.zeros(B, self.Hg, N, 128, **bf) for _ in range(self.G)]
        f32 = dict(dtype=torch.float32, device=device)
        self.rstd = [torch.zeros(B, self.Hg, N, **f32) for _ in range(self.G)]
        self.dinv = [torch.zeros(B, self.Hg, N, **f32) for _ in range(self.G)]
        self.lse = [torch.zeros(B, self.Hg * self.Gq, N, **f32) for _ in range(self.G)]
        self.flags = [torch.zeros(B * self.Hg * self.NB, dtype=torch.int32, device=device) for _ in range(self.G)]
        self.status = torch.zeros(64, dtype=torch.int32, device=device)
        self.o = torch.empty(B, self.C, Hq, D, **bf)

    # ---- helpers ----
    def _st(self):
        return torch.cuda.current_stream(self.dev).cuda_stream

    def _rows(self, j):
        return slice(self.bounds[j], self.bounds[j + 1])

    def empty_chunk(self, heads, j):
        n = self.bounds[j + 1] - self.bounds[j]
        return torch.empty(self.B, heads, n, self.D, dtype=torch.bfloat16, device=self.dev)

    def _hs(self, g):
        return slice(g * self.Hg, (g + 1) * self.Hg)

    # ---- protocol steps ----
    def set_local(self, q, k):
        self.Kf[:, :, self._rows(self.r)] = k
        self.Qf[:, :, self._rows(self.r)] = q

    def own_keys(self):
        return self.Kf[:, :, self._rows(self.r)].contiguous()

    def store_keys(self, j, buf):
        self.Kf[:, :, self._rows(j)] = buf

    def prep(self):
        lib = self.lib
        for g in range(self.G):
            kv = self.Kf[:, self._hs(g)]
            args = (kv.data_ptr(), kv.stride(0), kv.stride(1), kv.stride(2), self.khat[g].data_ptr(),
                    self.u[g].data_ptr(), self.rstd[g].data_ptr(), self.dinv[g].data_ptr(), self._st())
            _lib.check(lib.lucid_cp_prep(self.B, self.Hg, self.N, self.D, self.s, self.eps, 0, self.blk_lo, 1,
                                         *args), "lucid_cp_prep")
            _lib.check(lib.lucid_cp_prep(self.B, self.Hg, self.N, self.D, self.s, self.eps, self.blk_lo,
                                         self.blk_hi, 0, *args), "lucid_cp_prep")

    def store_values(self, g, j, buf):
        self.x[g][:, :, self._rows(j)] = buf
        _lib.check(self.lib.lucid_cp_publish(self.flags[g].data_ptr(), self.B * self.Hg, self.NB,
                                             self.bounds[j] // 128, self.bounds[j + 1] // 128, self._st()),
                   "lucid_cp_publish")

    def solve(self, g, v):
        vg = v[:, self._hs(g)]
        if vg.stride(-1) != 1:
            vg = vg.contiguous()
        # the kernel indexes V by global row: shift the pointer back by this rank's first row
        vptr = vg.data_ptr() - self.row0 * vg.stride(2) * vg.element_size()
        _lib.check(self.lib.lucid_cp_solve_fwd(self.B, self.Hg, self.N, self.D, self.s, self.blk_lo, self.blk_hi,
                                               self.max_ctas,
                                               vptr, vg.stride(0), vg.stride(1), vg.stride(2), self.x[g].data_ptr(),
                                               self.khat[g].data_ptr(), self.u[g].data_ptr(),
                                               self.dinv[g].data_ptr(), self.flags[g].data_ptr(),
                                               self.status.data_ptr(), self._st()), "lucid_cp_solve_fwd")
        self._vg = vg  # keep a contiguous copy alive until the kernel has run

    def own_values(self, g):
        return self.x[g][:, :, self._rows(self.r)].contiguous()

    def attend(self, g):
        hq = slice(g * self.Hg * self.Gq, (g + 1) * self.Hg * self.Gq)
        qg, kg = self.Qf[:, hq], self.Kf[:, self._hs(g)]
        og = self.o[:, :, hq].transpose(1, 2)   # [B, Hq_g, C, D] view of [B, C, Hq, D]
        optr = og.data_ptr() - self.row0 * og.stride(2) * og.element_size()
        _lib.check(self.lib.lucid_cp_attn_fwd(self.B, self.Hg * self.Gq, self.Hg, self.N, self.D, self.s, self.blk_lo,
                                              self.blk_hi, self.max_ctas, qg.data_ptr(), qg.stride(0), qg.stride(1), qg.stride(2),
                                              kg.data_ptr(), kg.stride(0), kg.stride(1), kg.stride(2),
                                              self.x[g].data_ptr(), optr, og.stride(0), og.stride(1), og.stride(2),
                                              self.lse[g].data_ptr(), self.status.data_ptr(), self._st()),
                   "lucid_cp_attn_fwd")

    def finish(self):
        self._check_status()
        return self.o

    def _check_status(self):
        st = int(self.status[0].item())
        if st != 0:
            raise _lib.LucidError(f"context-parallel kernels reported status {st:#x} (a bounded wait timed out)")

    # ---- backward ----
    def _hq(self, g):
        return slice(g * self.Hg * self.Gq, (g + 1) * self.Hg * self.Gq)

    def _shift(self, t, row_dim):
        """Address of global row 0 of a tensor holding this rank's rows (the
        kernels index outputs by global row)."""
        return t.data_ptr() - self.row0 * t.stride(row_dim) * t.element_size()

    def set_grad(self, do):
        B, N, D, Hq, H = self.B, self.N, self.D, self.Hq, self.H
        bf = dict(dtype=torch.bfloat16, device=self.dev)
        f32 = dict(dtype=torch.float32, device=self.dev)
        self.dOf = torch.zeros(B, Hq, N, D, **bf)
        self.dOf[:, :, self._rows(self.r)] = do.transpose(1, 2)
        self.delta = [torch.zeros(B, self.Hg * self.Gq, N, **f32) for _ in range(self.G)]
        for g in range(self.G):
            og = self.o[:, :, self._hq(g)].transpose(1, 2)
            dg = self.dOf[:, self._hq(g)]
            _lib.check(self.lib.lucid_cp_delta(B, self.Hg * self.Gq, N, D, self.row0, self.row0 + self.C,
                                               self._shift(og, 2), og.stride(0), og.stride(1), og.stride(2),
                                               dg.data_ptr(), dg.stride(0), dg.stride(1), dg.stride(2),
                                               self.delta[g].data_ptr(), self._st()), "lucid_cp_delta")
        # per-parity scratch of the head group in flight (group g uses g % 2)
        self.dx32 = [torch.empty(B, self.Hg, N, D, **f32) for _ in range(2)]
        self.dka32 = [torch.empty(B, self.Hg, N, D, **f32) for _ in range(2)]
        self.dkcol = [torch.empty(B, self.Hg, N, D, **f32) for _ in range(2)]
        self.dkrow = [torch.empty(B, self.Hg, N, D, **f32) for _ in range(2)]
        self.dvint = [torch.zeros(B, self.Hg, N, D, **bf) for _ in range(2)]
        self.bflags = [torch.zeros(B * self.Hg * self.NB, dtype=torch.int32, device=self.dev) for _ in range(self.G)]
        self.dq = torch.empty(B, Hq, self.C, D, **bf)
        self.dk = torch.empty(B, H, self.C, D, **bf)
        self.dv = torch.empty(B, H, self.C, D, **bf)

    def _own_stats(self, lst):
        return torch.cat([t[:, :, self._rows(self.r)] for t in lst], dim=1)

    def own_grad_inputs(self):
        rows = self._rows(self.r)
        packed = torch.cat([self.Qf[:, :, rows], self.dOf[:, :, rows], self.Kf[:, :, rows]], dim=1).contiguous()
        stats = torch.stack([self._own_stats(self.lse), self._own_stats(self.delta)]).contiguous()
        return [packed, stats]

    def empty_grad_inputs(self, j):
        n = self.bounds[j + 1] - self.bounds[j]
        return [torch.empty(self.B, 2 * self.Hq + self.H, n, self.D, dtype=torch.bfloat16, device=self.dev),
                torch.empty(2, self.B, self.Hq, n, dtype=torch.float32, device=self.dev)]

    def store_grad_inputs(self, j, bufs):
        packed, stats = bufs
        rows, Hq = self._rows(j), self.Hq
        self.Qf[:, :, rows] = packed[:, :Hq]
        self.dOf[:, :, rows] = packed[:, Hq:2 * Hq]
        self.Kf[:, :, rows] = packed[:, 2 * Hq:]
        for g in range(self.G):
            self.lse[g][:, :, rows] = stats[0][:, self._hq(g)]
            self.delta[g][:, :, rows] = stats[1][:, self._hq(g)]

    def prep_later(self):
        if self.blk_hi >= self.NB:
            return
        for g in range(self.G):
            kv = self.Kf[:, self._hs(g)]
            _lib.check(self.lib.lucid_cp_prep(self.B, self.Hg, self.N, self.D, self.s, self.eps, self.blk_hi,
                                              self.NB, 1, kv.data_ptr(), kv.stride(0), kv.stride(1), kv.stride(2),
                                              self.khat[g].data_ptr(), self.u[g].data_ptr(),
                                              self.rstd[g].data_ptr(), self.dinv[g].data_ptr(), self._st()),
                       "lucid_cp_prep")

    def _attn_bwd(self, g, passes):
        hq, pr = self._hq(g), g % 2
        qg, kg, dg = self.Qf[:, hq], self.Kf[:, self._hs(g)], self.dOf[:, hq]
        dq = self.dq[:, hq]
        _lib.check(self.lib.lucid_cp_attn_bwd(
            self.B, self.Hg * self.Gq, self.Hg, self.N, self.D, self.s, self.blk_lo, self.blk_hi, self.max_ctas,
            passes, qg.data_ptr(), qg.stride(0), qg.stride(1), qg.stride(2),
            kg.data_ptr(), kg.stride(0), kg.stride(1), kg.stride(2), self.x[g].data_ptr(),
            dg.data_ptr(), dg.stride(0), dg.stride(1), dg.stride(2), self.lse[g].data_ptr(),
            self.delta[g].data_ptr(), self._shift(dq, 2), dq.stride(0), dq.stride(1), dq.stride(2),
            self.dka32[pr].data_ptr(), self.dx32[pr].data_ptr(), self.status.data_ptr(), self._st()),
            "lucid_cp_attn_bwd")

    def _solve_bwd(self, g, passes):
        hs, pr = self._hs(g), g % 2
        kg, dk, dv = self.Kf[:, hs], self.dk[:, hs], self.dv[:, hs]
        _lib.check(self.lib.lucid_cp_solve_bwd(
            self.B, self.Hg, self.N, self.D, self.s, self.blk_lo, self.blk_hi, self.max_ctas, passes,
            kg.data_ptr(), kg.stride(0), kg.stride(1), kg.stride(2), self.x[g].data_ptr(),
            self.khat[g].data_ptr(), self.u[g].data_ptr(), self.rstd[g].data_ptr(), self.dinv[g].data_ptr(),
            self.dx32[pr].data_ptr(), self.dka32[pr].data_ptr(), self.dvint[pr].data_ptr(),
            self.dkcol[pr].data_ptr(), self.dkrow[pr].data_ptr(), self.bflags[g].data_ptr(),
            self._shift(dk, 2), dk.stride(0), dk.stride(1), dk.stride(2),
            self._shift(dv, 2), dv.stride(0), dv.stride(1), dv.stride(2), self.status.data_ptr(), self._st()),
            "lucid_cp_solve_bwd")

    def attn_col(self, g):
        self._attn_bwd(g, 1)

    def store_dv(self, g, j, buf):
        self.dvint[g % 2][:, :, self._rows(j)] = buf
        _lib.check(self.lib.lucid_cp_publish(self.bflags[g].data_ptr(), self.B * self.Hg, self.NB,
                                             self.bounds[j] // 128, self.bounds[j + 1] // 128, self._st()),
                   "lucid_cp_publish")

    def solve_col(self, g):
        self._solve_bwd(g, 1)

    def own_dv(self, g):
        return self.dvint[g % 2][:, :, self._rows(self.r)].contiguous()

    def rows(self, g):
        self._solve_bwd(g, 2)
        self._attn_bwd(g, 2)

    def finish_grad(self):
        self._check_status()
        return self.dq, self.dk, self.dv


class CPLucidAttentionFunction(torch.autograd.Function):
    """Autograd of the context-parallel op: the forward chain, then the
    backward chain with the forward's per-rank state (held by the protocol)."""

    @staticmethod
    def forward(ctx, q, k, v, proto):
        ctx.proto = proto
        return proto.run(q, k, v)

    @staticmethod
    def backward(ctx, do):
        proto, ctx.proto = ctx.proto, None
        dq, dk, dv = proto.backward(do.contiguous())
        return dq, dk, dv, None


def _protocol(q, k, v, group, scale, eps, head_groups, reserve_sms, bounds):
    W = dist.get_world_size(group) if dist.is_initialized() else 1
    r = dist.get_rank(group) if dist.is_initialized() else 0
    B, Hq, C, D = q.shape
    H = k.shape[1]
    s = D ** -0.5 if scale is None else scale
    if bounds is None:
        bounds = even_bounds(C * W, W)
    if bounds[r + 1] - bounds[r] != C:
        raise ValueError(f"rank {r} passed {C} rows but owns [{bounds[r]}, {bounds[r + 1]})")
    be = KernelBackend(B, H, Hq, bounds, D, s, eps, r, W, head_groups, q.device, reserve_sms)
    return ChunkProtocol(be, group)


def cp_lucid_attention(q, k, v, group=None, scale=None, eps=1e-5, head_groups=8, reserve_sms=8, bounds=None):
    """LUCID attention over a sequence split across the ranks of ``group``, with
    autograd: the arguments and the result are those of
    cp_lucid_attention_forward, and backward() runs the backward chain
    (every rank must call backward, as every rank called forward)."""
    proto = _protocol(q, k, v, group, scale, eps, head_groups, reserve_sms, bounds)
    return CPLucidAttentionFunction.apply(q, k, v, proto)


def cp_lucid_attention_forward(q, k, v, group=None, scale=None, eps=1e-5, head_groups=8, reserve_sms=8,
                               bounds=None):
    """LUCID attention forward over a sequence split across the ranks of ``group``.

    Each rank passes its own chunk: q [B, Hq, C_r, D], k, v [B, H, C_r, D] (bf16,
    CUDA), rank r holding rows [bounds[r], bounds[r+1]) of the sequence
    (``bounds`` as from balanced_bounds / even_bounds; None: equal chunks).
    Returns this rank's rows of O as [B, C_r, Hq, D] (the layout of
    eager_lucid_attention_forward, modeling_lucid.py:546)."""
    return _protocol(q, k, v, group, scale, eps, head_groups, reserve_sms, bounds).run(q, k, v)
