"""Builds the CPU oracle (test infrastructure): oracle/libcpu_oracle.so.

gcc -O2 -ffp-contract=off -fopenmp: every product and sum is rounded as
written in cpu_oracle.c, fused multiply-adds only where fmaf() is called.
"""

from __future__ import annotations

import shutil
import subprocess
import sys
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
SOURCES = (ORACLE_DIR / "cpu_oracle.c", ORACLE_DIR / "trace_oracle.c")
LIBRARY = ORACLE_DIR / "libcpu_oracle.so"


def build(force: bool = False) -> Path:
    newest = max([src.stat().st_mtime for src in SOURCES] + [Path(__file__).stat().st_mtime])
    if not force and LIBRARY.exists() and LIBRARY.stat().st_mtime >= newest:
        return LIBRARY
    cc = shutil.which("gcc") or "gcc"
    command = [cc, "-O2", "-std=c11", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared",
               "-fvisibility=hidden", *[str(src) for src in SOURCES], "-o", str(LIBRARY), "-lm"]
    done = subprocess.run(command, capture_output=True, text=True)
    if done.returncode != 0:
        raise RuntimeError("CPU oracle build failed:\n" + " ".join(command) + "\n" + done.stderr)
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
