"""Build recipe for the CPU oracle: oracle/_build/libexfold_oracle.so.

gcc, -O2, no floating-point contraction and no fast-math, so that every
float operation in exfold_oracle.c is one IEEE binary32 operation.
"""

from __future__ import annotations

import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_build" / "libexfold_oracle.so"
SRC = HERE / "exfold_oracle.c"


def build(force: bool = False) -> Path:
    OUT.parent.mkdir(parents=True, exist_ok=True)
    if not force and OUT.is_file() and OUT.stat().st_mtime >= SRC.stat().st_mtime:
        return OUT
    cmd = ["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
           "-fvisibility=hidden", "-Wall", "-Wextra", "-o", str(OUT), str(SRC), "-lm"]
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(force=True))
