"""Place an unmodified copy of the reference's GPU code in baseline/_ref/ (git-ignored).

The reference checkout has neither setup.py nor pyproject.toml, so
``pip install --target baseline/_ref <checkout>`` refuses it ("not installable").
This script does what that install would have done for the two pieces bench.py
times on the GPU as comparators, copying the files byte for byte:

  modeling_lucid.py              LucidAttention (torch path: get_v_prime + SDPA)
  lucid_path/triton_code/*.py    the LUCID-Path Triton op (parallel_lucid_path_attention)
  LICENSE files

bench.py imports them from baseline/_ref/ (the checkout itself is not present on
the GPU box; baseline/_ref/ travels with the repository snapshot).

Usage:  python baseline/install_ref.py /path/to/LUCID
"""
from __future__ import annotations

import hashlib
import json
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
DEST = os.path.join(HERE, "_ref")


def main(argv) -> int:
    if len(argv) != 2:
        print(__doc__)
        return 2
    src = argv[1]
    files = ["modeling_lucid.py", "LICENSE"]
    tc = os.path.join("lucid_path", "triton_code")
    files += [os.path.join(tc, f) for f in sorted(os.listdir(os.path.join(src, tc)))
              if f.endswith(".py") or f == "LICENSE"]
    record = {}
    for rel in files:
        a, b = os.path.join(src, rel), os.path.join(DEST, rel)
        os.makedirs(os.path.dirname(b), exist_ok=True)
        shutil.copyfile(a, b)
        with open(b, "rb") as f:
            record[rel] = hashlib.sha256(f.read()).hexdigest()
    with open(os.path.join(DEST, "INSTALLED.json"), "w") as f:
        json.dump({"source": "saisuryadv/LUCID checkout, unmodified", "files": record}, f, indent=1)
    print(f"copied {len(files)} files into {DEST}")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
