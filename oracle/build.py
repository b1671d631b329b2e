"""Builds the oracle's C helper (oracle/libhy_synth.so, the counter-based weight generator).

Test infrastructure only; see oracle/hy_oracle.py.
"""

from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libhy_synth.so")
SRC = os.path.join(HERE, "synth.c")


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    subprocess.run(["gcc", "-O2", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off", "-o", LIB, SRC], check=True)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
