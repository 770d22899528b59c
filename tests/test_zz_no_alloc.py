"""lucid_solve_fwd_noalloc: the solve forward for callers that cannot call
cudaMalloc (for example a plugin inside an engine that owns all device
memory, or a path that cannot afford an allocation's implicit device
synchronisation).  It takes no workspace; its scratch is a fixed static
device array.  Its results must equal those of lucid_solve_fwd, which takes
a caller-allocated workspace, on consecutive calls that reuse the array, and
its status word (read back by lucid_solve_fwd_noalloc_status) must be clear.

This file is collected last so that a failure here never hides another test."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _solve(lib, torch, k, v, noalloc):
    from lucid_b200 import padded_len
    B, H, N, D = k.shape
    Np = padded_len(N)
    dev = k.device
    x = torch.empty(B, H, Np, D, dtype=torch.bfloat16, device=dev)
    khat = torch.empty_like(x)
    u = torch.empty(B, H, Np, 128, dtype=torch.bfloat16, device=dev)
    rstd = torch.empty(B, H, Np, dtype=torch.float32, device=dev)
    dinv = torch.empty_like(rstd)
    st = torch.cuda.current_stream().cuda_stream
    s = D ** -0.5
    args = (B, H, N, D, s, 1e-5, k.data_ptr(), *k.stride()[:3], v.data_ptr(), *v.stride()[:3],
            x.data_ptr(), khat.data_ptr(), u.data_ptr(), rstd.data_ptr(), dinv.data_ptr())
    if noalloc:
        rc = lib.lucid_solve_fwd_noalloc(*args, st)
        assert rc == 0
        # the call's run-time status word, kept in the static array until the next call
        word = torch.full((1,), -1, dtype=torch.int32, pin_memory=True)
        assert lib.lucid_solve_fwd_noalloc_status(word.data_ptr(), st) == 0
        torch.cuda.synchronize()
        assert int(word[0]) == 0
    else:
        ws = torch.empty(lib.lucid_solve_fwd_workspace_bytes(B, H, N, D), dtype=torch.uint8, device=dev)
        rc = lib.lucid_solve_fwd(*args, ws.data_ptr(), ws.numel(), st)
    assert rc == 0
    torch.cuda.synchronize()
    return x[:, :, :N].float().cpu().numpy(), dinv[:, :, :N].cpu().numpy()


def test_noalloc_solve_matches_workspace_solve_on_consecutive_calls(cuda_device):
    import torch
    from lucid_b200 import _lib
    lib = _lib.load()
    g = torch.Generator(device="cpu").manual_seed(11)
    for (B, H, N) in ((1, 2, 700), (2, 3, 1000)):  # two calls in a row reuse the static scratch
        k = (0.6 * torch.randn(B, H, 1, 128, generator=g) + 0.8 * torch.randn(B, H, N, 128, generator=g))
        v = torch.randn(B, H, N, 128, generator=g)
        k, v = k.to(cuda_device, torch.bfloat16), v.to(cuda_device, torch.bfloat16)
        x_ref, d_ref = _solve(lib, torch, k, v, noalloc=False)
        x_na, d_na = _solve(lib, torch, k, v, noalloc=True)
        assert np.all(np.isfinite(x_na))
        # the bf16 tolerance of the other tests, and (same kernels, same inputs) equality
        assert np.max(np.abs(x_na - x_ref) - (1e-2 + 2.0 ** -8 * np.abs(x_ref))) <= 0
        np.testing.assert_array_equal(x_na, x_ref)
        np.testing.assert_array_equal(d_na, d_ref)


def test_noalloc_rejects_sizes_beyond_its_buffer(cuda_device):
    import torch
    from lucid_b200 import _lib
    lib = _lib.load()
    # B * H * ceil(N / 128) = 1 * 129 * 128 blocks > 16384: rejected before any launch
    k = torch.zeros(8, dtype=torch.bfloat16, device=cuda_device)
    rc = lib.lucid_solve_fwd_noalloc(1, 129, 128 * 128, 128, 0.088, 1e-5, k.data_ptr(), 0, 0, 128,
                                     k.data_ptr(), 0, 0, 128, k.data_ptr(), k.data_ptr(), k.data_ptr(),
                                     k.data_ptr(), k.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 6
