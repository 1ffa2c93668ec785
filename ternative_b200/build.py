"""In-tree build of libtvb200.so (nvcc, sm_100a).  The built library sits next
to this file so it travels with the source tree; nothing is pip-installed."""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")


def build(jobs: int = 8, verbose: bool = False) -> str:
    out = subprocess.run(["make", "-C", CSRC, f"-j{jobs}"], capture_output=not verbose, text=True)
    if out.returncode != 0:
        raise RuntimeError("libtvb200 build failed:\n" + (out.stdout or "") + (out.stderr or ""))
    return os.path.join(HERE, "libtvb200.so")


if __name__ == "__main__":
    print(build(verbose=True))
