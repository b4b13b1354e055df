"""Build the oracle's C checkers (test infrastructure, never the product path).

* ``oracle/libfp4_linear_port.so`` from ``oracle/fp4_linear_port.c`` (this
  repo's plain-C restatement of the source-exact FP4 linear).
* ``oracle/_ref/libvnni_source.so`` compiled from the REFERENCE's own source
  file ``mosaicvm/bench/vnni_source_kernel.c`` when the reference checkout is
  present (``$MOSAIC_REFERENCE``, default: a ``reference`` checkout beside
  this repository), with the flags
  the reference uses (``mosaicvm/bench/vnni_source.py:31-32``).  The output
  goes to ``oracle/_ref/`` only; no reference source is copied.
"""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF = Path(os.environ.get("MOSAIC_REFERENCE", str(HERE.parent.parent / "reference")))
VNNI_SRC = REF / "mosaicvm" / "bench" / "vnni_source_kernel.c"
VNNI_LIB = HERE / "_ref" / "libvnni_source.so"
PORT_LIB = HERE / "libfp4_linear_port.so"


def build() -> dict:
    out = {}
    subprocess.run(["gcc", "-O3", "-shared", "-fPIC", "-fopenmp", "-ffp-contract=off",
                    str(HERE / "fp4_linear_port.c"), "-o", str(PORT_LIB)], check=True)
    out["port"] = str(PORT_LIB)
    if VNNI_SRC.exists():
        VNNI_LIB.parent.mkdir(exist_ok=True)
        subprocess.run(["gcc", "-O3", "-shared", "-fPIC", "-mavxvnni", "-fopenmp", "-ffp-contract=off",
                        str(VNNI_SRC), "-o", str(VNNI_LIB)], check=True)
        out["reference"] = str(VNNI_LIB)
    return out


if __name__ == "__main__":
    print(build())
