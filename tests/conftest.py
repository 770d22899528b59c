import glob
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU (sm_100a)")


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """List the deviations every parity check measured (tests/parity.py)."""
    import parity

    for line in parity.summary_lines():
        terminalreporter.write_line(line)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def load_golden(name: str) -> dict:
    """Fixture produced by tests/golden/make_golden.py from the reference.
    Inputs (q, k, v, do) are exact bf16 values, returned as float64."""
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
        d = {k: z[k] for k in z.files}
    for nm in ("q", "k", "v", "do"):
        if f"{nm}_bf16" in d:
            d[nm] = from_bf16_bits(d.pop(f"{nm}_bf16")).astype(np.float64)
    return d


ATTN_CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "*.npz"))
                    if not os.path.basename(p).startswith(("blockwise", "path", "decode")))
PATH_CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "path_*.npz")))
DECODE_CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "decode_*.npz")))


def load_decode_golden(name: str) -> dict:
    """Decode fixture from tests/golden/make_golden.py (the reference's
    get_new_v_prime in float64).  Inputs are exact bf16 values."""
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
        d = {k: z[k] for k in z.files}
    for nm in ("k_cache", "x_cache", "k_new", "v_new"):
        d[nm] = from_bf16_bits(d.pop(f"{nm}_bf16")).astype(np.float64)
    return d


PATH_ATTN_CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "pathattn_*.npz")))


def load_path_golden(name: str) -> dict:
    """LUCID-Path fixture from tests/golden/make_path_golden.py (the reference
    Triton op, float32).  Inputs are exact bf16 values, returned as float64."""
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
        d = {k: z[k] for k in z.files}
    for nm in ("q", "k", "v", "w", "beta", "do"):
        if f"{nm}_bf16" in d:
            d[nm] = from_bf16_bits(d.pop(f"{nm}_bf16")).astype(np.float64)
    d.setdefault("q", None)
    return d


@pytest.fixture(scope="session")
def cuda_device():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
