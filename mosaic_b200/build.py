"""Build ``libmosaic_moe.so`` in-tree for sm_100a (``python -m mosaic_b200.build``).

Runs ``make`` in ``mosaic_b200/csrc`` (nvcc ``-gencode arch=compute_100a,code=sm_100a``
``-lineinfo``).  nvcc cross-compiles, so this works on hosts without a GPU.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent / "csrc"


def build(verbose: bool = False) -> Path:
    env = dict(os.environ)
    env.setdefault("NVCC", "/usr/local/cuda/bin/nvcc")
    jobs = str(min(8, os.cpu_count() or 1))
    out = subprocess.run(["make", "-C", str(CSRC), "-j", jobs], env=env, capture_output=not verbose, text=True)
    if out.returncode != 0:
        raise RuntimeError(f"mosaic_b200 build failed:\n{out.stdout}\n{out.stderr}")
    lib = CSRC.parent / "libmosaic_moe.so"
    if not lib.exists():
        raise RuntimeError(f"build finished but {lib} is missing")
    return lib


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
