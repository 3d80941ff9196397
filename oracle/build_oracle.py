"""Build recipe for the CPU oracle shared library (test infrastructure only).

    python oracle/build_oracle.py        # -> oracle/liboracle.so

Flags: -O3 -fopenmp for a multi-threaded CPU baseline; -ffp-contract=off so
every a*b+c is two IEEE roundings (the numpy restatement matches bit for bit);
-march=x86-64-v3 (AVX2/FMA ISA, no contraction) so the library also runs on
the GPU hosts, which receive this prebuilt file.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
SOURCES = [os.path.join(HERE, "tq_oracle.c"), os.path.join(HERE, "tq_oracle_polar.c")]


def build(force: bool = False) -> str:
    newest = max(os.path.getmtime(s) for s in SOURCES if os.path.exists(s))
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= newest:
        return LIB
    cmd = ["gcc", "-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fno-math-errno",
           "-fopenmp", "-fPIC", "-shared", "-std=gnu11", "-o", LIB + ".tmp"]
    cmd += [s for s in SOURCES if os.path.exists(s)]
    cmd += ["-lm"]
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
