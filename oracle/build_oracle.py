"""Builds the C oracle (``lthc_oracle.c``) into ``oracle/liblthc_oracle.so``.

Test infrastructure only.  The flags target x86-64-v3 (AVX2 + FMA) so the
library built in one container also loads on the GPU hosts, and disable
floating-point contraction so that only the explicit ``fmaf`` calls fuse.
"""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "lthc_oracle.c"
OUT = HERE / "liblthc_oracle.so"

CFLAGS = ["-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-fPIC", "-shared", "-std=c11"]


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and OUT.exists() and OUT.stat().st_mtime >= SRC.stat().st_mtime:
        return OUT
    cc = "gcc"  # the system compiler; a CC override may lack OpenMP
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [cc, *CFLAGS, "-o", str(tmp), str(SRC), "-lm"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force=True, verbose=True))
