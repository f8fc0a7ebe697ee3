"""Build the reference-side test programs into oracle/_ref/ (test infrastructure).

    python -m oracle.build_ref [--reference <reference root>]

The reference root comes from --reference, else $Q4_REFERENCE_ROOT, else a
`reference` checkout beside this repository.

`session_seam`: the reference's own session state machine
(FPGA_Project/software/qmap_prompt_demo/qot_session.c), compiled with gcc from
the reference sources where they lie, linked with oracle/session_seam_main.c
and libq4gpu.so (q4gpu_run_token as the runner).  Needs the reference tree
(present in the development container only); the binary lands in oracle/_ref/
and travels with the repository snapshot.  Nothing is copied from the
reference.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
OUT = HERE / "_ref"
LIB_DIR = REPO / "llm_accelerator_b200" / "_lib"


def reference_root() -> Path | None:
    """The reference checkout: $Q4_REFERENCE_ROOT, else a `reference` directory
    beside this repository's; None when neither exists."""
    env = os.environ.get("Q4_REFERENCE_ROOT")
    cand = Path(env) if env else REPO.parent / "reference"
    return cand if cand.is_dir() else None


def build_session_seam(ref: Path) -> Path | None:
    demo = ref / "FPGA_Project" / "software" / "qmap_prompt_demo"
    runtime = ref / "FPGA_Project" / "software" / "qmap_one_token_runtime"
    src = demo / "qot_session.c"
    if not src.exists() or not (LIB_DIR / "libq4gpu.so").exists():
        return None
    OUT.mkdir(exist_ok=True)
    exe = OUT / "session_seam"
    cc = shutil.which("gcc") or "gcc"
    cmd = [cc, "-O2", "-std=c11", "-Wall", "-I", str(demo), "-I", str(runtime), "-I", str(REPO / "include"),
           str(HERE / "session_seam_main.c"), str(src), "-L", str(LIB_DIR), "-lq4gpu",
           "-Wl,-rpath,$ORIGIN/../../llm_accelerator_b200/_lib", "-o", str(exe)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"session_seam build failed:\n{res.stdout}\n{res.stderr}")
    return exe


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, default=None)
    a = ap.parse_args()
    ref = a.reference or reference_root()
    exe = build_session_seam(ref) if ref else None
    print(exe if exe else "reference sources or libq4gpu.so missing: nothing built", file=sys.stderr)


if __name__ == "__main__":
    main()
