"""Float64 CPU backend of the context-parallel protocol (lucid_b200/cp.py) —
TEST INFRASTRUCTURE ONLY.  Implements the same per-segment steps as
KernelBackend with dense torch math (the oracle's formulas,
modeling_lucid.py:551-574, :505-549 and the analytic backward of :314-382)
so that the protocol can run on gloo ranks without a GPU.  Every step
asserts that the data it depends on has arrived: a schedule that computed
from a missing segment fails here instead of producing a wrong answer."""
import math

import torch


class CpuBackend:
    def __init__(self, B, H, Hq, layout, D, scale, eps, rank, world, head_groups):
        N = layout.N
        self.layout = layout
        self.B, self.H, self.Hq, self.N, self.D = B, H, Hq, N, D
        self.s, self.eps = scale, eps
        self.r, self.W = rank, world
        self.G, self.Hg, self.Gq = head_groups, H // head_groups, Hq // H
        self.C = layout.local_rows(rank)
        f = dict(dtype=torch.float64)
        self.Kf = torch.zeros(B, H, N, D, **f)
        self.Qf = torch.zeros(B, Hq, N, D, **f)
        self.x = [torch.zeros(B, self.Hg, N, D, **f) for _ in range(self.G)]
        self.keys_have = set()
        self.solved = [set() for _ in range(self.G)]   # segments whose X is present, per group
        self.o = torch.zeros(B, self.C, Hq, D, **f)
        self.lse = torch.zeros(B, Hq, N, **f)

    # ---- helpers ----
    def _rows(self, s):
        return slice(self.layout.lo(s), self.layout.hi(s))

    def _local(self, s):
        off = self.layout.local_offset(s)
        return slice(off, off + self.layout.hi(s) - self.layout.lo(s))

    def _hs(self, g):
        return slice(g * self.Hg, (g + 1) * self.Hg)

    def _hq(self, g):
        return slice(g * self.Hg * self.Gq, (g + 1) * self.Hg * self.Gq)

    def _e(self, a, b):
        return torch.exp(self.s * a @ b.transpose(-1, -2) - 1 / self.s)

    def empty_chunk(self, heads, s):
        return torch.empty(self.B, heads, self.layout.hi(s) - self.layout.lo(s), self.D, dtype=torch.float64)

    # ---- forward ----
    def set_local(self, q, k):
        for s in self.layout.mine(self.r):
            self.Kf[:, :, self._rows(s)] = k[:, :, self._local(s)]
            self.Qf[:, :, self._rows(s)] = q[:, :, self._local(s)]
            self.keys_have.add(s)

    def keys(self, s):
        return self.Kf[:, :, self._rows(s)].contiguous()

    def store_keys(self, s, buf):
        self.Kf[:, :, self._rows(s)] = buf
        self.keys_have.add(s)

    def prep(self):
        last = self.layout.mine(self.r)[-1]
        assert self.keys_have >= set(range(last + 1)), "prep before every earlier segment's keys arrived"
        k = self.Kf[:, :, : self.layout.hi(last)]
        self.khat = k / torch.sqrt((k * k).mean(-1, keepdim=True) + self.eps)

    def store_values(self, g, s, buf):
        self.x[g][:, :, self._rows(s)] = buf
        self.solved[g].add(s)

    def solve(self, t, g, v):
        assert self.solved[g] >= set(range(t)), "solve before every earlier segment arrived"
        c0, c1 = self.layout.lo(t), self.layout.hi(t)
        kh = self.khat[:, self._hs(g)]
        R = v[:, self._hs(g), self._local(t)].clone()
        if c0 > 0:
            R = R - self._e(kh[:, :, c0:c1], kh[:, :, :c0]) @ self.x[g][:, :, :c0]
        P = torch.tril(self._e(kh[:, :, c0:c1], kh[:, :, c0:c1]))
        self.x[g][:, :, c0:c1] = torch.linalg.solve_triangular(P, R, upper=False)
        self.solved[g].add(t)

    def own_values(self, t, g):
        return self.x[g][:, :, self._rows(t)].contiguous()

    def attend(self, t, g):
        assert self.solved[g] >= set(range(t + 1))
        c0, c1 = self.layout.lo(t), self.layout.hi(t)
        hq = self._hq(g)
        q = self.Qf[:, hq, c0:c1]
        k = self.Kf[:, self._hs(g), :c1].repeat_interleave(self.Gq, dim=1)
        x = self.x[g][:, :, :c1].repeat_interleave(self.Gq, dim=1)
        s = self.s * q @ k.transpose(-1, -2)
        s = s.masked_fill(torch.arange(c1)[None, :] > torch.arange(c0, c1)[:, None], -math.inf)
        self.o[:, self._local(t), hq] = (torch.softmax(s, -1) @ x).transpose(1, 2)
        self.lse[:, hq, c0:c1] = torch.logsumexp(s, -1)

    def finish(self):
        return self.o

    # ---- backward: every gradient of this rank's rows, from what has arrived ----
    def set_grad(self, do):
        f = dict(dtype=torch.float64)
        B, Hq, N, D = self.B, self.Hq, self.N, self.D
        self.dOf = torch.zeros(B, Hq, N, D, **f)
        self.delta = torch.zeros(B, Hq, N, **f)
        for s in self.layout.mine(self.r):
            d_s = do[:, self._local(s)]
            self.dOf[:, :, self._rows(s)] = d_s.transpose(1, 2)
            self.delta[:, :, self._rows(s)] = (d_s * self.o[:, self._local(s)]).sum(-1).transpose(1, 2)
        self.got = set(self.layout.mine(self.r))
        self.dvf = [torch.zeros(B, self.Hg, N, D, **f) for _ in range(self.G)]
        self.dv_got = [set() for _ in range(self.G)]
        self.dxo = {}
        self.dka = {}
        self.dkcol = {}
        self.dq = torch.zeros(B, Hq, self.C, D, **f)
        self.dk = torch.zeros(B, self.H, self.C, D, **f)
        self.dv = torch.zeros(B, self.H, self.C, D, **f)

    def grad_inputs(self, s):
        rows = self._rows(s)
        return [torch.cat([self.Qf[:, :, rows], self.dOf[:, :, rows], self.Kf[:, :, rows]], 1).contiguous(),
                torch.stack([self.lse[:, :, rows], self.delta[:, :, rows]]).contiguous()]

    def empty_grad_inputs(self, s):
        n = self.layout.hi(s) - self.layout.lo(s)
        return [torch.empty(self.B, 2 * self.Hq + self.H, n, self.D, dtype=torch.float64),
                torch.empty(2, self.B, self.Hq, n, dtype=torch.float64)]

    def store_grad_inputs(self, s, bufs):
        packed, stats = bufs
        rows, Hq = self._rows(s), self.Hq
        self.Qf[:, :, rows] = packed[:, :Hq]
        self.dOf[:, :, rows] = packed[:, Hq:2 * Hq]
        self.Kf[:, :, rows] = packed[:, 2 * Hq:]
        self.lse[:, :, rows] = stats[0]
        self.delta[:, :, rows] = stats[1]
        self.got.add(s)

    def prep_later(self):
        first = self.layout.mine(self.r)[0]
        assert self.got >= set(range(first, self.layout.n)), "backward inputs of a later segment missing"
        k = self.Kf
        self.rstd = 1 / torch.sqrt((k * k).mean(-1, keepdim=True) + self.eps)
        self.khat = k * self.rstd

    def attn_col(self, t, g):
        """dX and the attention's dK of segment t's key rows, over all later query rows."""
        c0, c1, N = self.layout.lo(t), self.layout.hi(t), self.N
        hq, hs = self._hq(g), self._hs(g)
        q, do = self.Qf[:, hq, c0:], self.dOf[:, hq, c0:]
        k = self.Kf[:, hs, c0:c1].repeat_interleave(self.Gq, dim=1)
        x = self.x[g][:, :, c0:c1].repeat_interleave(self.Gq, dim=1)
        mask = torch.arange(c0, N)[:, None] >= torch.arange(c0, c1)[None, :]
        p = torch.exp(self.s * q @ k.transpose(-1, -2) - self.lse[:, hq, c0:, None]) * mask
        ds = p * (do @ x.transpose(-1, -2) - self.delta[:, hq, c0:, None])
        B, Gq, Hg = self.B, self.Gq, self.Hg
        self.dxo[t, g] = (p.transpose(-1, -2) @ do).reshape(B, Hg, Gq, c1 - c0, self.D).sum(2)
        self.dka[t, g] = (self.s * ds.transpose(-1, -2) @ q).reshape(B, Hg, Gq, c1 - c0, self.D).sum(2)

    def store_dv(self, g, s, buf):
        self.dvf[g][:, :, self._rows(s)] = buf
        self.dv_got[g].add(s)

    def solve_col(self, t, g):
        """dV = P^-T dX of segment t's rows (needs dV of every later row) and the
        column part of dK^ (all later rows)."""
        assert self.dv_got[g] >= set(range(t + 1, self.layout.n)), "transposed solve before every later dV arrived"
        c0, c1 = self.layout.lo(t), self.layout.hi(t)
        kh, dvf = self.khat[:, self._hs(g)], self.dvf[g]
        R = self.dxo[t, g] - self._e(kh[:, :, c1:], kh[:, :, c0:c1]).transpose(-1, -2) @ dvf[:, :, c1:]
        P = torch.tril(self._e(kh[:, :, c0:c1], kh[:, :, c0:c1]))
        dvf[:, :, c0:c1] = torch.linalg.solve_triangular(P.transpose(-1, -2), R, upper=True)
        self.dv_got[g].add(t)
        mask = torch.arange(c0, self.N)[:, None] >= torch.arange(c0, c1)[None, :]
        dg = self.s * self._e(kh[:, :, c0:], kh[:, :, c0:c1]) * mask * \
            -(dvf[:, :, c0:] @ self.x[g][:, :, c0:c1].transpose(-1, -2))
        self.dkcol[t, g] = dg.transpose(-1, -2) @ kh[:, :, c0:]

    def own_dv(self, t, g):
        return self.dvf[g][:, :, self._rows(t)].contiguous()

    def rows(self, t, g):
        """Row part of dK^ and dQ of segment t's rows (all earlier columns), then
        dK through the RMSNorm."""
        c0, c1 = self.layout.lo(t), self.layout.hi(t)
        hs, hq = self._hs(g), self._hq(g)
        loc = self._local(t)
        kh, x, dv = self.khat[:, hs], self.x[g], self.dvf[g][:, :, c0:c1]
        mask = torch.arange(c0, c1)[:, None] >= torch.arange(c1)[None, :]
        dg = self.s * self._e(kh[:, :, c0:c1], kh[:, :, :c1]) * mask * -(dv @ x[:, :, :c1].transpose(-1, -2))
        dkh = self.dkcol[t, g] + dg @ kh[:, :, :c1]
        kho = kh[:, :, c0:c1]
        proj = (kho * dkh).sum(-1, keepdim=True) / self.D
        self.dk[:, hs, loc] = self.rstd[:, hs, c0:c1] * (dkh - proj * kho) + self.dka[t, g]
        self.dv[:, hs, loc] = dv
        q, do = self.Qf[:, hq, c0:c1], self.dOf[:, hq, c0:c1]
        k = self.Kf[:, hs, :c1].repeat_interleave(self.Gq, dim=1)
        xr = x[:, :, :c1].repeat_interleave(self.Gq, dim=1)
        p = torch.exp(self.s * q @ k.transpose(-1, -2) - self.lse[:, hq, c0:c1, None]) * mask
        ds = p * (do @ xr.transpose(-1, -2) - self.delta[:, hq, c0:c1, None])
        self.dq[:, hq, loc] = self.s * ds @ k

    def finish_grad(self):
        return self.dq, self.dk, self.dv
