"""Build the oracle's C restatement: ``oracle/_build/libvco.so``.

Test infrastructure only (the checker and the timed CPU baseline).  The
reference itself (Rust) cannot be compiled in this image: there is no cargo
or rustc and no crate registry, so there is no ``oracle/_ref``.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_build")
LIB = os.path.join(OUT, "libvco.so")


def build(force: bool = False) -> str:
    src = os.path.join(HERE, "vco.c")
    hdr = os.path.join(HERE, "..", "include", "vcommit.h")
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(src), os.path.getmtime(hdr)):
        return LIB
    os.makedirs(OUT, exist_ok=True)
    # No -march=native: the library also runs on the GPU host's CPU; OpenSSL
    # picks SHA-NI at run time.
    # -ffp-contract=off: every f64 product and sum rounds on its own, as in Rust.
    cmd = ["gcc", "-O3", "-ffp-contract=off", "-fPIC", "-shared", "-pthread", src, "-o", LIB + ".tmp",
           "-lcrypto", "-lm"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stderr}")
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
