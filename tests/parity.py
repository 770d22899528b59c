"""Parity bars shared by the GPU tests, and the record of measured deviations that
conftest.py prints at the end of a run.

The bar (bf16 outputs against a float32 / float64 reference value r):

  strict:   |ours - r| <= atol + ulp_bf16(r) / 2        atol = 1e-2 (x sqrt(G) for sums over G
                                                        grouped query heads)
            A bf16 number cannot come closer to r than half a bf16 ulp, so this is the
            "max-abs 1e-2" bar applied to the value before its final rounding to bf16.
            (|ours - bf16(r)| <= 1e-2 cannot hold above 2: one bf16 ulp there is 2^-6.)
  legacy:   |ours - r| <= atol + 2^-8 |r|               the earlier, looser bound, kept as a
                                                        second check (2^-8 |r| lies between
                                                        half and one ulp).

Every check records max |ours - r|, max |ours - bf16(r)| and the strict excess
(max |ours - r| - ulp/2), which the terminal summary lists per tensor.
"""
from __future__ import annotations

import math

import numpy as np

ATOL = 1e-2
RTOL_LEGACY = 2.0 ** -8

RECORDS: list[tuple[str, str, float, float, float, float]] = []


def half_ulp_bf16(a: np.ndarray) -> np.ndarray:
    """Half the spacing of bf16 numbers (8 significant bits) at |a|."""
    _, e = np.frexp(np.abs(a))          # |a| = m 2^e, m in [0.5, 1)
    return np.ldexp(1.0, e.astype(np.int64) - 9)


def round_bf16(a: np.ndarray) -> np.ndarray:
    """Round float values to the nearest bf16 (ties to even), returned as float64."""
    x = np.asarray(a, dtype=np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    b = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return b.astype(np.uint32).view(np.float32).astype(np.float64)


def check(ours, ref, case: str, what: str, group: int = 1, strict: bool = True) -> float:
    """Assert the bars above for one tensor (numpy arrays) and record the deviations.
    Returns max |ours - ref|."""
    ours = np.asarray(ours, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert ours.shape == ref.shape, f"{case} {what}: shape {ours.shape} vs {ref.shape}"
    assert np.all(np.isfinite(ours)), f"{case} {what}: non-finite values"
    err = np.abs(ours - ref)
    atol = ATOL * math.sqrt(group)
    hu = half_ulp_bf16(np.maximum(np.abs(ours), np.abs(ref)))
    strict_excess = float(np.max(err - hu))
    legacy_excess = float(np.max(err - (atol + RTOL_LEGACY * np.abs(ref))))
    max_abs = float(err.max())
    vs_bf16 = float(np.max(np.abs(ours - round_bf16(ref))))
    RECORDS.append((case, what, max_abs, vs_bf16, strict_excess, float(np.abs(ref).max())))
    assert legacy_excess <= 0, f"{case} {what}: legacy bound exceeded by {legacy_excess:.3e} (max abs {max_abs:.3e})"
    if strict:
        assert strict_excess <= atol, (f"{case} {what}: |ours - ref| - ulp/2 = {strict_excess:.3e} > {atol:.3e} "
                                       f"(max abs {max_abs:.3e})")
    return max_abs


def check_torch(ours, ref, case: str, what: str, group: int = 1, strict: bool = True) -> float:
    """check() for large torch tensors, evaluated on their device in float64."""
    import torch

    ours = ours.detach().to(torch.float64)
    ref = ref.detach().to(ours.device, torch.float64)
    assert ours.shape == ref.shape, f"{case} {what}: shape {tuple(ours.shape)} vs {tuple(ref.shape)}"
    assert bool(torch.isfinite(ours).all()), f"{case} {what}: non-finite values"
    err = (ours - ref).abs()
    atol = ATOL * math.sqrt(group)
    _, e = torch.frexp(torch.maximum(ours.abs(), ref.abs()))
    hu = torch.ldexp(torch.ones_like(err), e - 9)
    strict_excess = float((err - hu).max())
    legacy_excess = float((err - (atol + RTOL_LEGACY * ref.abs())).max())
    max_abs = float(err.max())
    vs_bf16 = float((ours - ref.to(torch.float32).to(torch.bfloat16).to(torch.float64)).abs().max())
    RECORDS.append((case, what, max_abs, vs_bf16, strict_excess, float(ref.abs().max())))
    assert legacy_excess <= 0, f"{case} {what}: legacy bound exceeded by {legacy_excess:.3e} (max abs {max_abs:.3e})"
    if strict:
        assert strict_excess <= atol, (f"{case} {what}: |ours - ref| - ulp/2 = {strict_excess:.3e} > {atol:.3e} "
                                       f"(max abs {max_abs:.3e})")
    return max_abs


def summary_lines() -> list[str]:
    if not RECORDS:
        return []
    agg: dict[tuple[str, str], list] = {}
    for case, what, a, b, c, m in RECORDS:
        cur = agg.setdefault((case, what), [0.0, 0.0, -np.inf, 0.0, 0])
        cur[0], cur[1], cur[2], cur[3] = max(cur[0], a), max(cur[1], b), max(cur[2], c), max(cur[3], m)
        cur[4] += 1
    out = ["parity: case tensor (checks) max|ours-ref| max|ours-bf16(ref)| max(|ours-ref|-ulp/2)<=1e-2 max|ref|"]
    for (case, what), (a, b, c, m, n) in agg.items():
        out.append(f"  {case:<22s} {what:<9s} ({n:3d}) {a:.3e} {b:.3e} {c:.3e} {m:.2e}")
    return out
