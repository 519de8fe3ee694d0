"""Build recipe for the CPU oracle (test infrastructure only).

Compiles ``oracle/dd_oracle.c`` with gcc into two shared libraries next to
this file: a portable x86-64 build and an x86-64-v3 (AVX2/FMA) build; the
loader in ``oracle/__init__.py`` picks the v3 build when the host CPU has
AVX2, FMA and BMI2. ``-ffp-contract=off`` keeps every a*b+c unfused, as in
the Rust reference. The reference itself (Rust + candle) cannot be compiled
in this image, so there is no ``oracle/_ref`` build.
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "dd_oracle.c"
VARIANTS = {
    "liboracle_generic.so": ["-march=x86-64", "-mtune=generic"],
    "liboracle_v3.so": ["-march=x86-64-v3", "-mtune=generic"],
}


def build(force: bool = False) -> list[Path]:
    out = []
    for name, flags in VARIANTS.items():
        lib = HERE / name
        if force or not lib.exists() or lib.stat().st_mtime < SRC.stat().st_mtime:
            cmd = ["gcc", "-O3", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
                   "-pthread", *flags, str(SRC), "-o", str(lib), "-lm"]
            subprocess.run(cmd, check=True)
        out.append(lib)
    return out


if __name__ == "__main__":
    for p in build(force="--force" in sys.argv):
        print(p)
