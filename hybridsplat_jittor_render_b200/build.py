"""Builds ``lib/libhybridsplat_rasterizer.so`` in-tree for sm_100a.

The library exports the C ABI declared in ``include/hybridsplat_rasterizer_c_api.h``.
CUDA sources are compiled with ``-gencode arch=compute_100a,code=sm_100a``.
Numeric compile flags are part of the results' definition:

* ``precise.cu`` uses ``--fmad=false`` like the reference's precise kernels;
  all of its arithmetic is explicitly rounded anyway.
* ``flashgs.cu`` / ``standard.cu`` write every rounding step explicitly
  (``csrc/fp.cuh``); ``expf`` is the only library math they call.
* Host ``.cpp`` files use ``-ffp-contract=off`` and no ``-march`` flag, so the
  host FP32 math rounds every operation like the reference's x86-64 build.

Usage: ``python -m hybridsplat_jittor_render_b200.build [--force] [--jobs N]``.
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_DIR = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
LIB_DIR = PACKAGE_DIR / "lib"
OBJ_DIR = PACKAGE_DIR / "lib" / "obj"
LIBRARY = LIB_DIR / "libhybridsplat_rasterizer.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_COMMON = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "--ftz=false",
    "--prec-div=true",
    "--prec-sqrt=true",
    "-Xcompiler=-fPIC",
    "-Xcompiler=-fvisibility=hidden",
    "-DHS_RASTERIZER_BUILDING_LIBRARY=1",
    *ARCH,
]
CXX_COMMON = [
    "-O2",
    "-std=c++17",
    "-fPIC",
    "-fvisibility=hidden",
    "-ffp-contract=off",
    "-Wall",
    "-Wextra",
    "-DHS_RASTERIZER_BUILDING_LIBRARY=1",
]

# (source, language, extra flags)
SOURCES = [
    ("flashgs.cu", "cuda", []),
    ("standard.cu", "cuda", []),
    ("standard_noalloc.cu", "cuda", []),
    ("sort.cu", "cuda", []),
    ("trace.cu", "cuda", []),
    ("view.cu", "cuda", []),
    ("pair_check.cu", "cuda", []),
    ("precise.cu", "cuda", ["--fmad=false"]),
    ("precise_exp.cu", "cuda", []),
    ("postprocess.cu", "cuda", []),
    ("c_api.cpp", "cxx", []),
    ("comm.cpp", "cxx", []),
    ("host_math.cpp", "cxx", []),
    ("workspace.cpp", "cxx", []),
]


def cuda_home() -> Path:
    return Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def _run(job: tuple[list[str], str]) -> str:
    command, label = job
    done = subprocess.run(command, capture_output=True, text=True)
    if done.returncode != 0:
        raise RuntimeError(f"build step failed ({label}):\n{' '.join(command)}\n{done.stdout}{done.stderr}")
    return done.stderr


def _inputs() -> list[Path]:
    files = [CSRC / name for name, _, _ in SOURCES]
    files += sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h"))
    files += sorted(INCLUDE.glob("*.h")) + [Path(__file__)]
    return files


def up_to_date() -> bool:
    if not LIBRARY.exists():
        return False
    built = LIBRARY.stat().st_mtime
    return all(p.stat().st_mtime <= built for p in _inputs())


def build(force: bool = False, jobs: int = 8, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIBRARY
    home = cuda_home()
    nvcc = str(home / "bin" / "nvcc")
    cxx = shutil.which("g++") or "g++"
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    includes = [f"-I{INCLUDE}", f"-I{CSRC}", f"-I{home / 'include'}"]
    steps = []
    objects = []
    for name, language, extra in SOURCES:
        obj = OBJ_DIR / (name + ".o")
        objects.append(obj)
        if language == "cuda":
            command = [nvcc, *CUDA_COMMON, *extra, *includes, "-c", str(CSRC / name), "-o", str(obj)]
            if verbose:
                command.insert(1, "-Xptxas=-v")
        else:
            command = [cxx, *CXX_COMMON, *extra, *includes, "-c", str(CSRC / name), "-o", str(obj)]
        steps.append((command, name))
    with concurrent.futures.ThreadPoolExecutor(max_workers=jobs) as pool:
        for log in pool.map(_run, steps):
            if verbose and log:
                print(log, file=sys.stderr)
    tmp = LIBRARY.with_suffix(".so.tmp")
    link = [nvcc, "-shared", *ARCH, *[str(o) for o in objects], "-o", str(tmp),
            f"-L{home / 'lib64'}", "-lcudart", "-lcublas", "-lcusolver", "-ldl"]
    _run((link, "link"))
    tmp.replace(LIBRARY)
    return LIBRARY


def main() -> int:
    parser = argparse.ArgumentParser(description="build the sm_100a HybridSplat rasterizer library")
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--jobs", type=int, default=8)
    parser.add_argument("--verbose", action="store_true", help="print ptxas register/spill reports")
    args = parser.parse_args()
    print(build(force=args.force, jobs=args.jobs, verbose=args.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
