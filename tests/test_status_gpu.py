"""Failure detection without a GPU fault: a kernel whose cross-CTA dependency never
arrives ends its bounded wait (2 s), records the failure in its status word and returns;
the context stays usable and the host raises LucidError from the word.

The wait is made to run out by the solve forward over row blocks [2, 4) of a block range
whose earlier blocks (0 and 1) nothing publishes: their flags stay zero."""
import time

import pytest

pytestmark = pytest.mark.gpu


def test_unpublished_dependency_times_out_with_status(cuda_device):
    import torch
    from lucid_b200 import _lib, solve_fwd
    lib = _lib.load()
    B, H, N = 1, 2, 512                                  # four row blocks per head
    g = torch.Generator(device="cpu").manual_seed(5)
    k = torch.randn(B, H, N, 128, generator=g).to(cuda_device, torch.bfloat16)
    v = torch.randn(B, H, N, 128, generator=g).to(cuda_device, torch.bfloat16)
    s = 128 ** -0.5
    x, khat, u, rstd, dinv = solve_fwd(k, v, s, 1e-5)
    _lib.check_status()                                  # the normal solve reported nothing
    flags = torch.zeros(B * H * 4, dtype=torch.int32, device=cuda_device)
    status = torch.zeros(64, dtype=torch.int32, device=cuda_device)
    x2 = torch.zeros_like(x)
    st = torch.cuda.current_stream().cuda_stream
    torch.cuda.synchronize()
    t0 = time.monotonic()
    rc = lib.lucid_cp_solve_fwd(B, H, N, 128, s, 2, 4, 0, v.data_ptr(), *v.stride()[:3], x2.data_ptr(),
                                khat.data_ptr(), u.data_ptr(), dinv.data_ptr(), flags.data_ptr(),
                                status.data_ptr(), st)
    assert rc == 0
    torch.cuda.synchronize()
    waited = time.monotonic() - t0
    word = int(status[0])
    assert word & 0xFF == 2, _lib.decode_status(word)            # a dependency flag never arrived
    assert (word >> 20) & 0xFF == 1, _lib.decode_status(word)    # in the solve forward
    assert 1.5 < waited < 60
    # the context is still usable: the same solve again gives the same values
    x3 = solve_fwd(k, v, s, 1e-5)[0]
    torch.cuda.synchronize()
    assert torch.equal(x3, x)
    # the host-side reader turns the word into an error naming kernel and cause
    _lib.STATUS.watch(status.view(torch.uint8), "lucid_cp_solve_fwd")
    with pytest.raises(_lib.LucidError, match="solve forward: a cross-CTA dependency flag never arrived"):
        _lib.check_status()
    _lib.check_status()                                  # consumed: nothing pending afterwards
