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

    def finish(self):
        return self.o
