"""C ABI checks that need no GPU: the library loads, exports every symbol
declared in include/lucid_b200.h, and the host-only helpers behave."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "lucid_b200.h")


def declared_symbols():
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(lucid_[a-z0-9_]+)\s*\(", txt)))


@pytest.fixture(scope="module")
def lib():
    from lucid_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        from lucid_b200 import build
        build.build()
    return _lib.load()


def test_header_declares_the_stage_entry_points():
    syms = declared_symbols()
    for s in ("lucid_solve_fwd", "lucid_attn_fwd", "lucid_attn_bwd", "lucid_solve_bwd"):
        assert s in syms


def test_library_exports_every_declared_symbol(lib):
    for s in declared_symbols():
        assert hasattr(lib, s), s


def test_binding_covers_every_declared_symbol():
    from lucid_b200 import _lib
    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_host_helpers(lib):
    assert lib.lucid_version() >= 100
    assert lib.lucid_padded_len(1) == 128
    assert lib.lucid_padded_len(128) == 128
    assert lib.lucid_padded_len(130) == 256
    assert lib.lucid_workspace_status_offset() == 0
    B, H, N, D = 2, 4, 1000, 128
    ws_f = lib.lucid_solve_fwd_workspace_bytes(B, H, N, D)
    assert ws_f >= 256 + B * H * 8 * 4
    ws_b = lib.lucid_solve_bwd_workspace_bytes(B, H, N, D)
    assert ws_b >= B * H * 1024 * 128 * (2 + 4 + 4)
    # attention backward scratch: status word + delta rows (no dQ accumulator: the row pass owns dQ)
    assert lib.lucid_attn_bwd_workspace_bytes(B, 8, H, N, D) >= 256 + B * 8 * 1024 * 4
    # stored-tile schedule: one 32 KB bf16 tile per block pair on top of the base workspace
    # (attention: plus the residual tile of each diagonal block)
    nb = 8  # ceil(1000 / 128)
    extra_attn = lib.lucid_attn_bwd_fast_workspace_bytes(B, 8, H, N, D) - lib.lucid_attn_bwd_workspace_bytes(
        B, 8, H, N, D)
    assert extra_attn == B * 8 * (nb * (nb + 1) // 2 + nb) * 32768
    extra_solve = lib.lucid_solve_bwd_fast_workspace_bytes(B, H, N, D) - ws_b
    assert extra_solve == B * H * (nb * (nb - 1) // 2) * 32768
    # a single block has no off-diagonal pair: the solve needs nothing extra
    assert lib.lucid_solve_bwd_fast_workspace_bytes(1, 1, 100, D) == lib.lucid_solve_bwd_workspace_bytes(1, 1, 100, D)


def test_decode_step_shapes(lib):
    """The fused decode step covers one new token with 1 or 2 query heads per kv
    head and two new tokens without grouping; its workspace holds per-split sums
    (128 floats per new token) and softmax partials (130 per query slot)."""
    for (hq, hkv, ln), want in {(8, 8, 1): 1, (4, 2, 1): 1, (4, 4, 2): 1, (8, 1, 1): 0, (4, 4, 3): 0,
                                (4, 2, 2): 0, (3, 2, 1): 0, (4, 0, 1): 0}.items():
        assert lib.lucid_decode_step_fused(hq, hkv, ln) == want, (hq, hkv, ln)
    a = lib.lucid_decode_step_workspace_bytes(4, 8, 4, 1, 5000, 128) - 256
    b = lib.lucid_decode_step_workspace_bytes(4, 8, 4, 2, 5000, 128) - 256
    assert a > 0 and a % ((128 + 2 * 130) * 4) == 0 and b == 2 * a
    # a shape without a single-pass kernel is refused before any launch
    rc = lib.lucid_decode_step(1, 8, 1, 1, 16, 128, 0.088, 1e-5, *([16, 128, 128, 128] * 7), 16, 4096, None)
    assert rc == 1


def test_argument_errors_without_launch(lib):
    """Bad shapes / alignment / workspace are rejected before any CUDA call."""
    from lucid_b200 import _lib as L
    null = None
    # head dimension outside 1..128 (smaller ones are zero-padded rows of 128)
    for d in (0, 129, 256):
        rc = lib.lucid_solve_fwd(1, 1, 128, d, 0.125, 1e-5, 16, 128, 128, 128, 16, 128, 128, 128,
                                 16, 16, 16, 16, 16, 16, 4096, null)
        assert rc == 1
    # decode reads rows of D elements with 8-byte loads: D must be a multiple of 4
    rc = lib.lucid_decode_update(1, 1, 1, 16, 66, 0.125, 1e-5, 16, 64, 64, 64, 16, 64, 64, 64, 16, 64, 64, 64,
                                 16, 64, 64, 64, 16, 64, 64, 64, 16, 4096, null)
    assert rc == 1
    # more than 65535 (batch, head) rows in a decode grid
    rc = lib.lucid_decode_update(256, 256, 1, 16, 64, 0.125, 1e-5, 16, 64, 64, 64, 16, 64, 64, 64, 16, 64, 64, 64,
                                 16, 64, 64, 64, 16, 64, 64, 64, 16, 4096, null)
    assert rc == 1
    rc = lib.lucid_decode_attn(256, 256, 1, 1, 16, 64, 0.125, 16, 64, 64, 64, 16, 64, 64, 64, 16, 64, 64, 64,
                               16, 64, 64, 64, 16, 4096, null)
    assert rc == 1
    # misaligned pointer
    rc = lib.lucid_solve_fwd(1, 1, 128, 128, 0.088, 1e-5, 18, 128, 128, 128, 16, 128, 128, 128,
                             16, 16, 16, 16, 16, 16, 4096, null)
    assert rc == 2
    # workspace too small
    rc = lib.lucid_solve_fwd(1, 1, 128, 128, 0.088, 1e-5, 16, 128, 128, 128, 16, 128, 128, 128,
                             16, 16, 16, 16, 16, 16, 8, null)
    assert rc == 3
    # Hq not a multiple of Hkv
    rc = lib.lucid_attn_fwd(1, 3, 2, 128, 128, 0.088, 16, 128, 128, 128, 16, 128, 128, 128, 16,
                            16, 128, 128, 128, 16, None, 16, 4096, null)
    assert rc == 1
    # empty problems are a no-op
    rc = lib.lucid_solve_fwd(1, 1, 0, 128, 0.088, 1e-5, 16, 128, 128, 128, 16, 128, 128, 128,
                             16, 16, 16, 16, 16, 16, 4096, null)
    assert rc == 0
    with pytest.raises(L.LucidError):
        L.check(3, "x")


def test_ops_refuse_cpu_tensors():
    torch = pytest.importorskip("torch")
    from lucid_b200 import lucid_attention
    q = torch.zeros(1, 1, 128, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        lucid_attention(q, q, q)


def test_status_words_decode():
    from lucid_b200 import _lib
    assert _lib.decode_status(2 | (1 << 20)).startswith("solve forward: a cross-CTA dependency flag never arrived")
    msg = _lib.decode_status(1 | (0x12 << 8) | (4 << 20))
    assert msg.startswith("transposed-solve column pass: an mbarrier wait timed out")
    assert "0x90" in msg


def test_solve_fwd_chain_schedule_workspace(lib, monkeypatch):
    """The chain schedule's workspace (flags, 8 W slots of 64 KB, 3 E tiles of 32 KB per
    row block, per head) is asked for only when the library would run that schedule:
    few heads per GPU (here a CPU process, which models a 148-SM B200), or when forced."""
    monkeypatch.delenv("LUCID_B200_SOLVE_SCHEDULE", raising=False)
    N, D = 32768, 128
    nb = N // 128

    def extra(B, H):
        return (-(-(B * H * nb * 4) // 256) * 256 + B * H * 8 * 128 * 128 * 4 + B * H * nb * 3 * 128 * 128 * 2)

    base4 = lib.lucid_solve_fwd_workspace_bytes(1, 4, N, D)
    assert lib.lucid_solve_fwd_fast_workspace_bytes(1, 4, N, D) == base4 + extra(1, 4)   # 4 heads: chains
    base32 = lib.lucid_solve_fwd_workspace_bytes(1, 32, N, D)
    assert lib.lucid_solve_fwd_fast_workspace_bytes(1, 32, N, D) == base32              # 32 heads: wavefront
    # the layer forward sizes its workspace by the kv heads
    assert lib.lucid_fused_fwd_workspace_bytes(1, 32, 4, N, D) == base4 + extra(1, 4)
    monkeypatch.setenv("LUCID_B200_SOLVE_SCHEDULE", "wavefront")
    assert lib.lucid_solve_fwd_fast_workspace_bytes(1, 4, N, D) == base4
    monkeypatch.setenv("LUCID_B200_SOLVE_SCHEDULE", "chain")
    assert lib.lucid_solve_fwd_fast_workspace_bytes(1, 32, N, D) == base32 + extra(1, 32)
    # never more chains than the grid leaves room for workers
    assert lib.lucid_solve_fwd_fast_workspace_bytes(1, 200, 1024, D) == lib.lucid_solve_fwd_workspace_bytes(
        1, 200, 1024, D)


def test_fused_fwd_argument_errors(lib):
    """Shape and alignment errors come back before any CUDA call (no GPU needed)."""
    ok = ctypes.c_void_p(4096)   # 16-byte aligned dummies, never dereferenced
    bad = ctypes.c_void_p(4098)
    args = lambda q, o: (1, 4, 2, 256, 128, 0.1, 1e-5, q, 0, 0, 128, ok, 0, 0, 128, ok, 0, 0, 128,
                         ok, ok, ok, ok, ok, o, 0, 0, 128, ok, None, ok, 1 << 20, None)
    assert lib.lucid_fused_fwd(*args(bad, ok)) == 2            # LUCID_ERR_ALIGN
    assert lib.lucid_fused_fwd(*args(ok, bad)) == 2
    a = list(args(ok, ok))
    a[1], a[2] = 3, 2                                           # Hq not a multiple of Hkv
    assert lib.lucid_fused_fwd(*a) == 1                         # LUCID_ERR_SHAPE
    a = list(args(ok, ok))
    a[4] = 129                                                  # head_dim above 128
    assert lib.lucid_fused_fwd(*a) == 1
