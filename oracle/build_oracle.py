"""Compile the C restatement of the oracle (test infrastructure).

Output: oracle/_build/libq4oracle.so (git-ignored; travels with the tree).
"""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "q4_oracle.c"
OUT = HERE / "_build" / "libq4oracle.so"


def build(force: bool = False) -> Path:
    if not force and OUT.exists() and OUT.stat().st_mtime >= SRC.stat().st_mtime:
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    cc = shutil.which("gcc") or "cc"
    tmp = OUT.with_suffix(".so.tmp")
    # no FMA contraction: the float32 quantiser must round every step alone
    cmd = [cc, "-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared", str(SRC),
           "-o", str(tmp), "-lm"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    tmp.replace(OUT)
    return OUT


if __name__ == "__main__":
    print(build(force=True))
