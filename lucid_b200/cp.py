"""Context-parallel LUCID attention for long sequences (the 128K
configuration): one process per GPU, the sequence cut into row segments each
owned by one rank, forward and backward.

The reference runs long sequences on one GPU (the blockwise solver of
modeling_lucid.py:285-312 under gradient checkpointing); this module spreads
one sequence over the GPUs of a node.

Math.  X = P^-1 V is a forward substitution, so segment t needs the solved
values X_s and the keys K_s of every earlier segment s < t:
    R_t = V_t - sum_{s<t} exp(s K^_t K^_s^T - 1/s) X_s ,  X_t = P_tt^-1 R_t
and the attention of segment t's queries needs K_s and X_s of every s <= t.
In the backward a rank computes every gradient of its own rows: its column
passes (attention dX / dK over its own key blocks, the transposed solve
dV = P^-T dX and the column part of dK^) need the rows after each of its
segments; its row passes (dQ, the row part of dK^) only the rows before,
which the forward brought in.  No partial sums cross ranks.

Layouts (Layout): contiguous chunks (one segment per rank; even_bounds,
balanced_bounds, train_bounds) or zigzag (zigzag_layout: 2W equal segments,
rank r owning segments r and 2W-1-r).  With contiguous chunks the forward's
work (growing with the row) and the backward's column passes (shrinking with
it) cannot both be balanced; the zigzag pairs an early and a late segment on
every rank and balances each phase on its own.

Protocol (all point-to-point NCCL send/recv on one communicator per pair of
ranks, no collective):
  forward   1. every rank sends the raw keys of each of its segments to every
               rank owning a later segment (inputs: this starts at once);
            2. for each own segment t in sequence order and each kv-head group
               g in order, a rank receives X_s(g) of every foreign s < t,
               marks those row blocks solved (the wavefront solve's per-block
               flags), solves segment t, sends X_t(g) to every rank owning a
               later segment and runs the attention of t's queries for g;
  backward  the mirror image: q, dO, raw keys, lse and delta = rowsum(dO o O)
            of each own segment go to every rank owning an earlier segment;
            then for each own segment t in reverse sequence order and each
            group, dV_s(g) of every foreign s > t is received, the transposed
            solve of t runs, dV_t(g) goes to the ranks owning earlier
            segments, and t's row passes run.
NCCL matches a pair's sends and receives per direction in issue order, so on
every pair both ends keep one order: forward messages by (source segment,
group) ascending, backward messages by source segment descending then group
ascending.  A rank sends in that order by construction (it walks its own
segments and groups in that order) and posts each receive at its
segment's turn in the same walk, ahead of need.  Kernels
never wait on another launch: every cross-rank dependency is a stream-ordered
NCCL receive, and the persistent kernels leave `reserve_sms` SMs free so the
NCCL kernels run alongside.  The schedule is checked for deadlock freedom
with every rank's operations fully serialised (tests/test_cp_cpu.py).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib

__all__ = ["cp_lucid_attention_forward", "cp_lucid_attention", "ChunkProtocol", "KernelBackend", "Layout",
           "balanced_bounds", "even_bounds", "train_bounds", "zigzag_layout"]


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


class Layout:
    """The sequence rows [0, N) as segments in sequence order, segment s =
    rows [lo_s, hi_s) owned by rank owner_s.  A rank's local tensors hold its
    segments' rows concatenated in sequence order."""

    def __init__(self, segs):
        self.segs = [(int(lo), int(hi), int(o)) for lo, hi, o in segs]
        if not self.segs or self.segs[0][0] != 0 or any(
                self.segs[i][1] != self.segs[i + 1][0] for i in range(len(self.segs) - 1)):
            raise ValueError("segments must cover [0, N) in order")
        if any(hi <= lo for lo, hi, _ in self.segs):
            raise ValueError("empty segment")
        self.N = self.segs[-1][1]
        self.n = len(self.segs)

    @classmethod
    def contiguous(cls, bounds):
        return cls([(bounds[r], bounds[r + 1], r) for r in range(len(bounds) - 1)])

    def lo(self, s):
        return self.segs[s][0]

    def hi(self, s):
        return self.segs[s][1]

    def owner(self, s):
        return self.segs[s][2]

    def mine(self, r):
        return [s for s in range(self.n) if self.segs[s][2] == r]

    def local_rows(self, r):
        return sum(self.hi(s) - self.lo(s) for s in self.mine(r))

    def local_offset(self, s):
        """Row of segment s's first row in its owner's local tensors."""
        o = self.owner(s)
        return sum(self.hi(t) - self.lo(t) for t in range(s) if self.owner(t) == o)

    def later_owners(self, s, r):
        """Ranks other than r owning a segment after s (they need segment s's
        forward messages)."""
        return sorted({self.owner(t) for t in range(s + 1, self.n)} - {r})

    def earlier_owners(self, s, r):
        return sorted({self.owner(t) for t in range(s)} - {r})

    def check(self, align=256, world=None):
        if any(lo % align for lo, _, _ in self.segs) or self.N % 128:
            raise ValueError(f"segment bounds must sit on multiples of {align} rows (N a multiple of 128)")
        if world is not None and sorted({o for _, _, o in self.segs}) != list(range(world)):
            raise ValueError("every rank must own at least one segment")


def zigzag_layout(N: int, world: int, align: int = 256):
    """2W segments of (nearly) equal length, rank r owning segments r and
    2W-1-r: an early and a late segment per rank, so the forward's work
    (growing with the row) and the backward's column passes (shrinking with
    it) are both balanced."""
    n = 2 * world
    b = [int(round(N * i / n / align)) * align for i in range(n)] + [N]
    for i in range(1, n):
        b[i] = min(max(b[i], b[i - 1] + align), N - (n - i) * align)
    return Layout([(b[i], b[i + 1], i if i < world else n - 1 - i) for i in range(n)])


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
    """The message schedule of the forward and backward chains, independent of
    how the segments are computed (``backend``) and of the process group's
    device.  ``backend.layout`` is the Layout."""

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

    def _post(self, buf, src):
        if isinstance(buf, list):   # a message of several tensors, sent in list order
            return buf, _MultiReq([self._recv(b, src) for b in buf])
        return buf, self._recv(buf, src)

    def run(self, q, k, v):
        be, r = self.be, self.rank
        L = be.layout
        mine = L.mine(r)
        last = mine[-1]
        be.set_local(q, k)
        # Messages are issued in one global order, segment by segment in sequence
        # order: a rank sends its own segment's messages and posts the receives of a
        # foreign segment it needs (every segment before its last one) at that
        # segment's turn, so both ends of every pair issue their common messages in
        # the same order, whichever direction they flow.
        # 1. raw keys: segment s goes to every other rank owning a later segment
        sends, keys = [], {}
        for s in range(L.n):
            if L.owner(s) == r:
                for d in L.later_owners(s, r):
                    sends.append(self._send(be.keys(s), d))
            elif s < last:
                keys[s] = self._post(be.empty_chunk(be.H, s), L.owner(s))
        for s, (buf, rq) in keys.items():
            rq.wait()
            be.store_keys(s, buf)
        be.prep()
        # 2. solved values: an own segment is solved group by group, each X_t(g) sent
        #    to the ranks owning later segments; a foreign segment's X_s(g) receives
        #    are posted at its turn and waited right before the first solve needing them
        posted, stored = {}, set()
        for t in range(L.n):
            if L.owner(t) != r:
                if t < last:
                    for g in range(be.G):
                        posted[t, g] = self._post(be.empty_chunk(be.Hg, t), L.owner(t))
                continue
            for g in range(be.G):
                for s in range(t):
                    if L.owner(s) == r or (s, g) in stored:
                        continue
                    buf, rq = posted[s, g]
                    rq.wait()
                    be.store_values(g, s, buf)
                    stored.add((s, g))
                be.solve(t, g, v)
                xs = be.own_values(t, g)
                sends += [self._send(xs, d) for d in L.later_owners(t, r)]
                be.attend(t, g)
        for s_ in sends:
            s_.wait()
        return be.finish()

    def backward(self, do):
        """Gradients of this rank's rows after run(): returns what the
        backend's finish_grad returns (dq, dk, dv of the rank's rows).  The
        mirror image of run: segments walked from the last one down."""
        be, r = self.be, self.rank
        L = be.layout
        first = L.mine(r)[0]
        be.set_grad(do)
        # 1. q, dO, raw keys, lse and delta: segment s goes to every other rank
        #    owning an earlier segment
        sends, ins = [], {}
        for s in range(L.n - 1, -1, -1):
            if L.owner(s) == r:
                for d in L.earlier_owners(s, r):
                    sends += [self._send(t_, d) for t_ in be.grad_inputs(s)]
            elif s > first:
                ins[s] = self._post(be.empty_grad_inputs(s), L.owner(s))
        for s, (bufs, rq) in ins.items():
            rq.wait()
            be.store_grad_inputs(s, bufs)
        be.prep_later()
        # 2. dV, per own segment from the last one down and head group in order
        posted, stored = {}, set()
        for t in range(L.n - 1, -1, -1):
            if L.owner(t) != r:
                if t > first:
                    for g in range(be.G):
                        posted[t, g] = self._post(be.empty_chunk(be.Hg, t), L.owner(t))
                continue
            be.attn_col(t, 0)
            for g in range(be.G):
                for s in range(L.n - 1, t, -1):
                    if L.owner(s) == r or (s, g) in stored:
                        continue
                    buf, rq = posted[s, g]
                    rq.wait()
                    be.store_dv(g, s, buf)
                    stored.add((s, g))
                be.solve_col(t, g)
                dv = be.own_dv(t, g)
                sends += [self._send(dv, d) for d in L.earlier_owners(t, r)]
                if g + 1 < be.G:
                    be.attn_col(t, g + 1)
                be.rows(t, g)
        for s_ in sends:
            s_.wait()
        return be.finish_grad()


class _MultiReq:
    """Several receives waited as one (a message made of several tensors)."""

    def __init__(self, reqs):
        self.reqs = reqs

    def wait(self):
        for rq in self.reqs:
            rq.wait()


class KernelBackend:
    """The segment computations on the B200 kernels (C ABI lucid_cp_*)."""

    def __init__(self, B, H, Hq, layout, D, scale, eps, rank, world, head_groups, device, reserve_sms=8):
        if D != 128:
            raise NotImplementedError("head_dim must be 128")
        layout.check(256, world)
        if H % head_groups or Hq % H:
            raise ValueError("head_groups must divide the kv heads and Hq must be a multiple of H")
        N = layout.N
        self.layout = layout
        self.lib = _lib.load()
        self.B, self.H, self.Hq, self.N, self.D = B, H, Hq, N, D
        self.s, self.eps = float(scale), float(eps)
        self.r, self.W = rank, world
        self.G, self.Hg, self.Gq = head_groups, H // head_groups, Hq // H
        self.C = layout.local_rows(rank)
        self.NB = N // 128
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
        self.o_res = torch.empty_like(self.o)   # bf16 rounding residual of O (for rowsum(dO * O))

    # ---- helpers ----
    def _st(self):
        return torch.cuda.current_stream(self.dev).cuda_stream

    def _rows(self, s):
        return slice(self.layout.lo(s), self.layout.hi(s))

    def _local(self, s):
        off = self.layout.local_offset(s)
        return slice(off, off + self.layout.hi(s) - self.layout.lo(s))

    def _blk(self, s):
        return self.layout.lo(s) // 128, self.layout.hi(s) // 128

    def _shift(self, t, s, row_dim):
        """Address of global row 0 of a local tensor (this rank's rows in
        segment order) for the rows of segment s: the kernels index by global row."""
        delta = self.layout.local_offset(s) - self.layout.lo(s)
        return t.data_ptr() + delta * t.stride(row_dim) * t.element_size()

    def empty_chunk(self, heads, s):
        n = self.layout.hi(s) - self.layout.lo(s)
        return torch.empty(self.B, heads, n, self.D, dtype=torch.bfloat16, device=self.dev)

    def _hs(self, g):
        return slice(g * self.Hg, (g + 1) * self.Hg)

    def _hq(self, g):
        return slice(g * self.Hg * self.Gq, (g + 1) * self.Hg * self.Gq)

    def _check_status(self):
        st = int(self.status[0].item())
        if st != 0:
            raise _lib.LucidError(f"context-parallel kernels reported status {st:#x} (a bounded wait timed out)")

    # ---- forward ----
    def set_local(self, q, k):
        for s in self.layout.mine(self.r):
            self.Kf[:, :, self._rows(s)] = k[:, :, self._local(s)]
            self.Qf[:, :, self._rows(s)] = q[:, :, self._local(s)]

    def keys(self, s):
        return self.Kf[:, :, self._rows(s)].contiguous()

    def store_keys(self, s, buf):
        self.Kf[:, :, self._rows(s)] = buf

    def _prep(self, s, khat_only):
        lo, hi = self._blk(s)
        for g in range(self.G):
            kv = self.Kf[:, self._hs(g)]
            _lib.check(self.lib.lucid_cp_prep(self.B, self.Hg, self.N, self.D, self.s, self.eps, lo, hi, khat_only,
                                              kv.data_ptr(), kv.stride(0), kv.stride(1), kv.stride(2),
                                              self.khat[g].data_ptr(), self.u[g].data_ptr(), self.rstd[g].data_ptr(),
                                              self.dinv[g].data_ptr(), self._st()), "lucid_cp_prep")

    def prep(self):
        L, mine = self.layout, self.layout.mine(self.r)
        for s in range(mine[-1] + 1):
            if L.owner(s) == self.r:
                self._prep(s, 0)
            else:
                self._prep(s, 1)   # received keys: k^ only

    def store_values(self, g, s, buf):
        self.x[g][:, :, self._rows(s)] = buf
        lo, hi = self._blk(s)
        _lib.check(self.lib.lucid_cp_publish(self.flags[g].data_ptr(), self.B * self.Hg, self.NB, lo, hi,
                                             self._st()), "lucid_cp_publish")

    def solve(self, t, g, v):
        vg = v[:, self._hs(g)]
        if vg.stride(-1) != 1:
            vg = vg.contiguous()
        lo, hi = self._blk(t)
        _lib.check(self.lib.lucid_cp_solve_fwd(self.B, self.Hg, self.N, self.D, self.s, lo, hi, self.max_ctas,
                                               self._shift(vg, t, 2), vg.stride(0), vg.stride(1), vg.stride(2),
                                               self.x[g].data_ptr(), self.khat[g].data_ptr(), self.u[g].data_ptr(),
                                               self.dinv[g].data_ptr(), self.flags[g].data_ptr(),
                                               self.status.data_ptr(), self._st()), "lucid_cp_solve_fwd")
        self._vg = vg  # keep a contiguous copy alive until the kernel has run

    def own_values(self, t, g):
        return self.x[g][:, :, self._rows(t)].contiguous()

    def attend(self, t, g):
        hq = self._hq(g)
        qg, kg = self.Qf[:, hq], self.Kf[:, self._hs(g)]
        og = self.o[:, :, hq].transpose(1, 2)   # [B, Hq_g, C, D] view of [B, C, Hq, D]
        orr = self.o_res[:, :, hq].transpose(1, 2)
        lo, hi = self._blk(t)
        _lib.check(self.lib.lucid_cp_attn_fwd(self.B, self.Hg * self.Gq, self.Hg, self.N, self.D, self.s, lo, hi,
                                              self.max_ctas, qg.data_ptr(), qg.stride(0), qg.stride(1), qg.stride(2),
                                              kg.data_ptr(), kg.stride(0), kg.stride(1), kg.stride(2),
                                              self.x[g].data_ptr(), self._shift(og, t, 2), og.stride(0), og.stride(1),
                                              og.stride(2), self.lse[g].data_ptr(), self._shift(orr, t, 2),
                                              self.status.data_ptr(), self._st()), "lucid_cp_attn_fwd")

    def finish(self):
        self._check_status()
        return self.o

    # ---- backward ----
    def set_grad(self, do):
        B, N, D, Hq, H = self.B, self.N, self.D, self.Hq, self.H
        bf = dict(dtype=torch.bfloat16, device=self.dev)
        f32 = dict(dtype=torch.float32, device=self.dev)
        mine = self.layout.mine(self.r)
        self.dOf = torch.zeros(B, Hq, N, D, **bf)
        for s in mine:
            self.dOf[:, :, self._rows(s)] = do[:, self._local(s)].transpose(1, 2)
        self.delta = [torch.zeros(B, self.Hg * self.Gq, N, **f32) for _ in range(self.G)]
        for g in range(self.G):
            og = self.o[:, :, self._hq(g)].transpose(1, 2)
            orr = self.o_res[:, :, self._hq(g)].transpose(1, 2)
            dg = self.dOf[:, self._hq(g)]
            for s in mine:
                _lib.check(self.lib.lucid_cp_delta(B, self.Hg * self.Gq, N, D, self.layout.lo(s), self.layout.hi(s),
                                                   self._shift(og, s, 2), og.stride(0), og.stride(1), og.stride(2),
                                                   dg.data_ptr(), dg.stride(0), dg.stride(1), dg.stride(2),
                                                   self._shift(orr, s, 2), self.delta[g].data_ptr(), self._st()),
                           "lucid_cp_delta")
        # per-parity scratch of the head group in flight (group g uses g % 2); dV is kept
        # per group: a rank's earlier segment needs the dV its later segment solved
        self.dx32 = [torch.empty(B, self.Hg, N, D, **f32) for _ in range(2)]
        self.dka32 = [torch.empty(B, self.Hg, N, D, **f32) for _ in range(2)]
        self.dkcol = [torch.empty(B, self.Hg, N, D, **f32) for _ in range(2)]
        self.dkrow = [torch.empty(B, self.Hg, N, D, **f32) for _ in range(2)]
        self.dvint = [torch.zeros(B, self.Hg, N, D, **bf) for _ in range(self.G)]
        self.bflags = [torch.zeros(B * self.Hg * self.NB, dtype=torch.int32, device=self.dev) for _ in range(self.G)]
        self.dq = torch.empty(B, Hq, self.C, D, **bf)
        self.dk = torch.empty(B, H, self.C, D, **bf)
        self.dv = torch.empty(B, H, self.C, D, **bf)

    def _stats(self, lst, s):
        return torch.cat([t[:, :, self._rows(s)] for t in lst], dim=1)

    def grad_inputs(self, s):
        rows = self._rows(s)
        packed = torch.cat([self.Qf[:, :, rows], self.dOf[:, :, rows], self.Kf[:, :, rows]], dim=1).contiguous()
        stats = torch.stack([self._stats(self.lse, s), self._stats(self.delta, s)]).contiguous()
        return [packed, stats]

    def empty_grad_inputs(self, s):
        n = self.layout.hi(s) - self.layout.lo(s)
        return [torch.empty(self.B, 2 * self.Hq + self.H, n, self.D, dtype=torch.bfloat16, device=self.dev),
                torch.empty(2, self.B, self.Hq, n, dtype=torch.float32, device=self.dev)]

    def store_grad_inputs(self, s, bufs):
        packed, stats = bufs
        rows, Hq = self._rows(s), self.Hq
        self.Qf[:, :, rows] = packed[:, :Hq]
        self.dOf[:, :, rows] = packed[:, Hq:2 * Hq]
        self.Kf[:, :, rows] = packed[:, 2 * Hq:]
        for g in range(self.G):
            self.lse[g][:, :, rows] = stats[0][:, self._hq(g)]
            self.delta[g][:, :, rows] = stats[1][:, self._hq(g)]

    def prep_later(self):
        # the forward prepared every segment up to this rank's last one; the later
        # (foreign) segments' keys arrived with the backward's inputs: k^ only
        for s in range(self.layout.mine(self.r)[-1] + 1, self.layout.n):
            self._prep(s, 1)

    def _attn_bwd(self, t, g, passes):
        hq, pr = self._hq(g), g % 2
        qg, kg, dg = self.Qf[:, hq], self.Kf[:, self._hs(g)], self.dOf[:, hq]
        dq = self.dq[:, hq]
        lo, hi = self._blk(t)
        _lib.check(self.lib.lucid_cp_attn_bwd(
            self.B, self.Hg * self.Gq, self.Hg, self.N, self.D, self.s, lo, hi, self.max_ctas,
            passes, qg.data_ptr(), qg.stride(0), qg.stride(1), qg.stride(2),
            kg.data_ptr(), kg.stride(0), kg.stride(1), kg.stride(2), self.x[g].data_ptr(),
            dg.data_ptr(), dg.stride(0), dg.stride(1), dg.stride(2), self.lse[g].data_ptr(),
            self.delta[g].data_ptr(), self._shift(dq, t, 2), dq.stride(0), dq.stride(1), dq.stride(2),
            self.dka32[pr].data_ptr(), self.dx32[pr].data_ptr(), self.status.data_ptr(), self._st()),
            "lucid_cp_attn_bwd")

    def _solve_bwd(self, t, g, passes):
        hs, pr = self._hs(g), g % 2
        kg, dk, dv = self.Kf[:, hs], self.dk[:, hs], self.dv[:, hs]
        lo, hi = self._blk(t)
        _lib.check(self.lib.lucid_cp_solve_bwd(
            self.B, self.Hg, self.N, self.D, self.s, lo, hi, self.max_ctas, passes,
            kg.data_ptr(), kg.stride(0), kg.stride(1), kg.stride(2), self.x[g].data_ptr(),
            self.khat[g].data_ptr(), self.u[g].data_ptr(), self.rstd[g].data_ptr(), self.dinv[g].data_ptr(),
            self.dx32[pr].data_ptr(), self.dka32[pr].data_ptr(), self.dvint[g].data_ptr(),
            self.dkcol[pr].data_ptr(), self.dkrow[pr].data_ptr(), self.bflags[g].data_ptr(),
            self._shift(dk, t, 2), dk.stride(0), dk.stride(1), dk.stride(2),
            self._shift(dv, t, 2), dv.stride(0), dv.stride(1), dv.stride(2), self.status.data_ptr(), self._st()),
            "lucid_cp_solve_bwd")

    def attn_col(self, t, g):
        self._attn_bwd(t, g, 1)

    def store_dv(self, g, s, buf):
        self.dvint[g][:, :, self._rows(s)] = buf
        lo, hi = self._blk(s)
        _lib.check(self.lib.lucid_cp_publish(self.bflags[g].data_ptr(), self.B * self.Hg, self.NB, lo, hi,
                                             self._st()), "lucid_cp_publish")

    def solve_col(self, t, g):
        self._solve_bwd(t, g, 1)

    def own_dv(self, t, g):
        return self.dvint[g][:, :, self._rows(t)].contiguous()

    def rows(self, t, g):
        self._solve_bwd(t, g, 2)
        self._attn_bwd(t, g, 2)

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


def _layout_of(bounds, layout, C, W):
    if layout is not None:
        return layout
    return Layout.contiguous(bounds if bounds is not None else even_bounds(C * W, W))


def _protocol(q, k, v, group, scale, eps, head_groups, reserve_sms, bounds, layout):
    W = dist.get_world_size(group) if dist.is_initialized() else 1
    r = dist.get_rank(group) if dist.is_initialized() else 0
    B, Hq, C, D = q.shape
    H = k.shape[1]
    s = D ** -0.5 if scale is None else scale
    L = _layout_of(bounds, layout, C, W)
    if L.local_rows(r) != C:
        raise ValueError(f"rank {r} passed {C} rows but owns {L.local_rows(r)} (segments {L.mine(r)})")
    be = KernelBackend(B, H, Hq, L, D, s, eps, r, W, head_groups, q.device, reserve_sms)
    return ChunkProtocol(be, group)


def cp_lucid_attention(q, k, v, group=None, scale=None, eps=1e-5, head_groups=8, reserve_sms=8, bounds=None,
                       layout=None):
    """LUCID attention over a sequence split across the ranks of ``group``, with
    autograd: the arguments and the result are those of
    cp_lucid_attention_forward, and backward() runs the backward chain
    (every rank must call backward, as every rank called forward)."""
    proto = _protocol(q, k, v, group, scale, eps, head_groups, reserve_sms, bounds, layout)
    return CPLucidAttentionFunction.apply(q, k, v, proto)


def cp_lucid_attention_forward(q, k, v, group=None, scale=None, eps=1e-5, head_groups=8, reserve_sms=8,
                               bounds=None, layout=None):
    """LUCID attention forward over a sequence split across the ranks of ``group``.

    Each rank passes its own rows: q [B, Hq, C_r, D], k, v [B, H, C_r, D] (bf16,
    CUDA), the rows of its segments concatenated in sequence order.  ``layout``
    (a Layout, e.g. zigzag_layout) or ``bounds`` (contiguous chunk bounds as from
    balanced_bounds / train_bounds / even_bounds; default equal chunks) says which
    rows a rank owns.  Returns this rank's rows of O as [B, C_r, Hq, D] (the
    layout of eager_lucid_attention_forward, modeling_lucid.py:546)."""
    return _protocol(q, k, v, group, scale, eps, head_groups, reserve_sms, bounds, layout).run(q, k, v)
