"""Float64 CPU backend of the context-parallel protocol (lucid_b200/cp.py) —
TEST INFRASTRUCTURE ONLY.  Implements the same steps as KernelBackend with
dense torch math (the oracle's formulas, modeling_lucid.py:551-574 and
:505-549) so that the chunk protocol can run on gloo ranks without a GPU."""
import math

import torch


class CpuBackend:
    def __init__(self, B, H, Hq, bounds, D, scale, eps, rank, world, head_groups):
        N = bounds[-1]
        self.B, self.H, self.Hq, self.N, self.D = B, H, Hq, N, D
        self.s, self.eps = scale, eps
        self.r, self.W = rank, world
        self.G, self.Hg, self.Gq = head_groups, H // head_groups, Hq // H
        self.bounds = bounds
        self.C = bounds[rank + 1] - bounds[rank]
        f = dict(dtype=torch.float64)
        self.Kf = torch.zeros(B, H, N, D, **f)
        self.Qf = torch.zeros(B, Hq, N, D, **f)
        self.x = [torch.zeros(B, self.Hg, N, D, **f) for _ in range(self.G)]
        self.solved = [set() for _ in range(self.G)]
        self.o = torch.zeros(B, self.C, Hq, D, **f)
        self.lse = torch.zeros(B, Hq, N, **f)

    def _rows(self, j):
        return slice(self.bounds[j], self.bounds[j + 1])

    def _hs(self, g):
        return slice(g * self.Hg, (g + 1) * self.Hg)

    def empty_chunk(self, heads, j):
        return torch.empty(self.B, heads, self.bounds[j + 1] - self.bounds[j], self.D, dtype=torch.float64)

    def set_local(self, q, k):
        self.Kf[:, :, self._rows(self.r)] = k
        self.Qf[:, :, self._rows(self.r)] = q

    def own_keys(self):
        return self.Kf[:, :, self._rows(self.r)].contiguous()

    def store_keys(self, j, buf):
        self.Kf[:, :, self._rows(j)] = buf

    def prep(self):
        k = self.Kf[:, :, : self.bounds[self.r + 1]]
        self.khat = k / torch.sqrt((k * k).mean(-1, keepdim=True) + self.eps)

    def store_values(self, g, j, buf):
        self.x[g][:, :, self._rows(j)] = buf
        self.solved[g].add(j)

    def solve(self, g, v):
        assert self.solved[g] == set(range(self.r)), "solve before every earlier chunk arrived"
        c0, c1 = self.bounds[self.r], self.bounds[self.r + 1]
        kh = self.khat[:, self._hs(g)]
        R = v[:, self._hs(g)].clone()
        if c0 > 0:
            E = torch.exp(self.s * kh[:, :, c0:c1] @ kh[:, :, :c0].transpose(-1, -2) - 1 / self.s)
            R = R - E @ self.x[g][:, :, :c0]
        P = torch.tril(torch.exp(self.s * kh[:, :, c0:c1] @ kh[:, :, c0:c1].transpose(-1, -2) - 1 / self.s))
        self.x[g][:, :, c0:c1] = torch.linalg.solve_triangular(P, R, upper=False)

    def own_values(self, g):
        return self.x[g][:, :, self._rows(self.r)].contiguous()

    def attend(self, g):
        c0, c1 = self.bounds[self.r], self.bounds[self.r + 1]
        hq = slice(g * self.Hg * self.Gq, (g + 1) * self.Hg * self.Gq)
        q = self.Qf[:, hq, c0:c1]
        k = self.Kf[:, self._hs(g), :c1].repeat_interleave(self.Gq, dim=1)
        x = self.x[g][:, :, :c1].repeat_interleave(self.Gq, dim=1)
        s = self.s * q @ k.transpose(-1, -2)
        rows = torch.arange(c0, c1)[:, None]
        s = s.masked_fill(torch.arange(c1)[None, :] > rows, -math.inf)
        self.o[:, :, hq] = (torch.softmax(s, -1) @ x).transpose(1, 2)
        self.lse[:, hq, c0:c1] = torch.logsumexp(s, -1)

    def finish(self):
        return self.o

    # ---- backward: every gradient of this rank's rows, from what has arrived ----
    def _hq(self, g):
        return slice(g * self.Hg * self.Gq, (g + 1) * self.Hg * self.Gq)

    def _e(self, a, b):
        return torch.exp(self.s * a @ b.transpose(-1, -2) - 1 / self.s)

    def set_grad(self, do):
        f = dict(dtype=torch.float64)
        B, Hq, N, D = self.B, self.Hq, self.N, self.D
        self.dOf = torch.zeros(B, Hq, N, D, **f)
        self.delta = torch.zeros(B, Hq, N, **f)
        c0, c1 = self.bounds[self.r], self.bounds[self.r + 1]
        self.dOf[:, :, c0:c1] = do.transpose(1, 2)
        self.delta[:, :, c0:c1] = (do * self.o).sum(-1).transpose(1, 2)
        self.got = {self.r}
        self.dvf = [torch.zeros(B, self.Hg, N, D, **f) for _ in range(self.G)]
        self.dv_got = [set() for _ in range(self.G)]
        self.dxo = [None] * self.G
        self.dka = [None] * self.G
        self.dq = torch.zeros(B, Hq, self.C, D, **f)
        self.dk = torch.zeros(B, self.H, self.C, D, **f)
        self.dv = torch.zeros(B, self.H, self.C, D, **f)

    def own_grad_inputs(self):
        rows = self._rows(self.r)
        return [torch.cat([self.Qf[:, :, rows], self.dOf[:, :, rows], self.Kf[:, :, rows]], 1).contiguous(),
                torch.stack([self.lse[:, :, rows], self.delta[:, :, rows]]).contiguous()]

    def empty_grad_inputs(self, j):
        n = self.bounds[j + 1] - self.bounds[j]
        return [torch.empty(self.B, 2 * self.Hq + self.H, n, self.D, dtype=torch.float64),
                torch.empty(2, self.B, self.Hq, n, dtype=torch.float64)]

    def store_grad_inputs(self, j, bufs):
        packed, stats = bufs
        rows, Hq = self._rows(j), self.Hq
        self.Qf[:, :, rows] = packed[:, :Hq]
        self.dOf[:, :, rows] = packed[:, Hq:2 * Hq]
        self.Kf[:, :, rows] = packed[:, 2 * Hq:]
        self.lse[:, :, rows] = stats[0]
        self.delta[:, :, rows] = stats[1]
        self.got.add(j)

    def prep_later(self):
        assert self.got == set(range(self.r, self.W)), "backward inputs of a later chunk missing"
        k = self.Kf
        self.rstd = 1 / torch.sqrt((k * k).mean(-1, keepdim=True) + self.eps)
        self.khat = k * self.rstd

    def attn_col(self, g):
        """dX and the attention's dK of this rank's key rows, over all later query rows."""
        c0, c1, N = self.bounds[self.r], self.bounds[self.r + 1], self.N
        hq, hs = self._hq(g), self._hs(g)
        q, do = self.Qf[:, hq, c0:], self.dOf[:, hq, c0:]
        k = self.Kf[:, hs, c0:c1].repeat_interleave(self.Gq, dim=1)
        x = self.x[g][:, :, c0:c1].repeat_interleave(self.Gq, dim=1)
        mask = torch.arange(c0, N)[:, None] >= torch.arange(c0, c1)[None, :]
        p = torch.exp(self.s * q @ k.transpose(-1, -2) - self.lse[:, hq, c0:, None]) * mask
        ds = p * (do @ x.transpose(-1, -2) - self.delta[:, hq, c0:, None])
        B, Gq, Hg = self.B, self.Gq, self.Hg
        self.dxo[g] = (p.transpose(-1, -2) @ do).reshape(B, Hg, Gq, c1 - c0, self.D).sum(2)
        self.dka[g] = (self.s * ds.transpose(-1, -2) @ q).reshape(B, Hg, Gq, c1 - c0, self.D).sum(2)

    def store_dv(self, g, j, buf):
        self.dvf[g][:, :, self._rows(j)] = buf
        self.dv_got[g].add(j)

    def solve_col(self, g):
        """dV = P^-T dX of this rank's rows (needs dV of every later row) and the
        column part of dK^ (all later rows)."""
        assert self.dv_got[g] == set(range(self.r + 1, self.W)), "transposed solve before every later dV arrived"
        c0, c1 = self.bounds[self.r], self.bounds[self.r + 1]
        kh, dvf = self.khat[:, self._hs(g)], self.dvf[g]
        R = self.dxo[g] - self._e(kh[:, :, c1:], kh[:, :, c0:c1]).transpose(-1, -2) @ dvf[:, :, c1:]
        P = torch.tril(self._e(kh[:, :, c0:c1], kh[:, :, c0:c1]))
        dvf[:, :, c0:c1] = torch.linalg.solve_triangular(P.transpose(-1, -2), R, upper=True)
        mask = torch.arange(c0, self.N)[:, None] >= torch.arange(c0, c1)[None, :]
        dg = self.s * self._e(kh[:, :, c0:], kh[:, :, c0:c1]) * mask * \
            -(dvf[:, :, c0:] @ self.x[g][:, :, c0:c1].transpose(-1, -2))
        self.dkcol = dg.transpose(-1, -2) @ kh[:, :, c0:]

    def own_dv(self, g):
        return self.dvf[g][:, :, self._rows(self.r)].contiguous()

    def rows(self, g):
        """Row part of dK^ and dQ of this rank's rows (all earlier columns),
        then dK through the RMSNorm."""
        c0, c1 = self.bounds[self.r], self.bounds[self.r + 1]
        hs, hq = self._hs(g), self._hq(g)
        kh, x, dv = self.khat[:, hs], self.x[g], self.dvf[g][:, :, c0:c1]
        mask = torch.arange(c0, c1)[:, None] >= torch.arange(c1)[None, :]
        dg = self.s * self._e(kh[:, :, c0:c1], kh[:, :, :c1]) * mask * -(dv @ x[:, :, :c1].transpose(-1, -2))
        dkh = self.dkcol + dg @ kh[:, :, :c1]
        kho = kh[:, :, c0:c1]
        proj = (kho * dkh).sum(-1, keepdim=True) / self.D
        self.dk[:, hs] = self.rstd[:, hs, c0:c1] * (dkh - proj * kho) + self.dka[g]
        self.dv[:, hs] = dv
        q, do = self.Qf[:, hq, c0:c1], self.dOf[:, hq, c0:c1]
        k = self.Kf[:, hs, :c1].repeat_interleave(self.Gq, dim=1)
        xr = x[:, :, :c1].repeat_interleave(self.Gq, dim=1)
        p = torch.exp(self.s * q @ k.transpose(-1, -2) - self.lse[:, hq, c0:c1, None]) * mask
        ds = p * (do @ xr.transpose(-1, -2) - self.delta[:, hq, c0:c1, None])
        self.dq[:, hq] = self.s * ds @ k

    def finish_grad(self):
        return self.dq, self.dk, self.dv
