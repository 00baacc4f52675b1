"""Build recipe for the reference oracle libraries (test infrastructure only).

This script compiles the reference's OWN sources, in place under the
reference checkout, into ``oracle/_ref/``. Nothing from the reference is
copied into this repository. Two artefacts are produced:

``oracle/_ref/libref_hybridsplat.so``
    The reference native backend (``jittor_hybridsplat/ops/native``) rebuilt
    for Blackwell with the per-file numeric flags of its own CMake project
    (``jittor_hybridsplat/ops/native/CMakeLists.txt:109-127,165-169``; Release
    build type as chosen by ``jittor_hybridsplat/ops/build.py:273``). The
    OptiX backend cannot be built here (the OptiX SDK headers are absent), so
    ``oracle/ref_harness.cu`` supplies the one symbol ``c_api.cpp`` needs from
    it (``hs_optix_release_context``, ``optix/optix_backend.h:5``) plus
    diagnostic entry points that call the reference render kernels directly.
    The architecture is ``sm_100`` because ``--arch 100`` in the reference
    build driver becomes ``CMAKE_CUDA_ARCHITECTURES=100-real``
    (``jittor_hybridsplat/ops/build.py:320``).

``oracle/_ref/libref_prepare.so``
    The host-only FlashGS NPZ activation (``rasterizer/flashgs_prepare.cpp``)
    built with g++; it runs on any CPU and pins the host activation bit-exactly.

Usage: ``python oracle/build_ref.py [--reference PATH] [--jobs 8]``. The
reference checkout is ``--reference``, else the environment variable
``HYBRIDSPLAT_REFERENCE_ROOT``, else a directory named ``reference`` beside
the directory holding this repository. When it is absent the script does
nothing and exits 0; prebuilt ``oracle/_ref`` files are then used as they are.
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
OUT_DIR = ORACLE_DIR / "_ref"
REPO_DIR = ORACLE_DIR.parent


def default_reference() -> Path:
    """--reference default: $HYBRIDSPLAT_REFERENCE_ROOT, else ../reference
    beside the repository."""
    env = os.environ.get("HYBRIDSPLAT_REFERENCE_ROOT")
    return Path(env) if env else REPO_DIR.parent / "reference"

# Release-mode flags CMake adds for both languages (CMAKE_<LANG>_FLAGS_RELEASE).
_RELEASE = ["-O3", "-DNDEBUG"]
# Target-wide CUDA options (CMakeLists.txt:165-169) plus the C++17 standard
# (CMakeLists.txt:144-148) and hidden visibility (CMakeLists.txt:171-183).
_CUDA_COMMON = [
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "--ftz=false",
    "--prec-div=true",
    "--prec-sqrt=true",
    "-Xcompiler=-fPIC",
    "-Xcompiler=-fvisibility=hidden",
    "-gencode",
    "arch=compute_100,code=sm_100",
]
_CXX_COMMON = [
    "-std=c++17",
    "-fPIC",
    "-fvisibility=hidden",
    "-fvisibility-inlines-hidden",
]
_DEFINES = [
    "-DHS_RASTERIZER_BUILDING_LIBRARY=1",
    '-DHS_RASTERIZER_BUILD_ID="reference-oracle-sm100"',
]


def _native(reference: Path) -> Path:
    return reference / "jittor_hybridsplat" / "ops" / "native"


def _include_flags(native: Path, cuda_home: Path) -> list[str]:
    vendor = native / "vendor"
    dirs = [
        native / "include",
        native / "rasterizer",
        native / "optix",
        vendor / "flashgs",
        vendor / "flashgs" / "glm",
        vendor / "standard_rasterizer",
        vendor / "standard_glm",
        vendor / "optix_tracer",
        cuda_home / "include",
    ]
    return [f"-I{d}" for d in dirs]


def _sources(native: Path) -> list[tuple[Path, str, list[str]]]:
    """(source, language, per-file options) as in CMakeLists.txt:86-127."""
    r = native / "rasterizer"
    fg = native / "vendor" / "flashgs" / "cuda_rasterizer"
    std = native / "vendor" / "standard_rasterizer"
    fmad_off = ["--fmad=false"]
    return [
        (r / "c_api.cpp", "cxx", []),
        (r / "flashgs_backend.cu", "cuda", []),
        (r / "flashgs_prepare.cpp", "cxx", []),
        (r / "full_rasterizer.cu", "cuda", []),
        (fg / "preprocess.cu", "cuda", ["-O1", "-Xptxas=-O1"]),
        (fg / "render.cu", "cuda", ["-O1", "-Xptxas=-O1"]),
        (fg / "sort.cu", "cuda", ["-O1", "-Xptxas=-O1"]),
        (std / "forward.cu", "cuda", []),
        (r / "precise_camera_center.cu", "cuda", []),
        (r / "precise_direction.cu", "cuda", fmad_off),
        (r / "precise_disk_rotation.cu", "cuda", fmad_off),
        (r / "precise_exp.cu", "cuda", []),
        (r / "precise_matrix.cu", "cuda", []),
        (r / "precise_activation.cu", "cuda", ["--fmad=false", "--ftz=false"]),
        (r / "precise_reflection_trace.cu", "cuda", fmad_off),
        (r / "precise_sh.cu", "cuda", fmad_off),
        (ORACLE_DIR / "ref_harness.cu", "cuda", []),
    ]


def _compile(job: tuple[list[str], Path]) -> tuple[Path, str]:
    command, target = job
    completed = subprocess.run(command, capture_output=True, text=True)
    if completed.returncode != 0:
        raise RuntimeError(
            f"reference oracle compile failed for {target.name}:\n"
            + " ".join(command)
            + "\n"
            + completed.stdout
            + completed.stderr
        )
    return target, completed.stderr


def build(reference: Path | None = None, jobs: int = 8, force: bool = False) -> bool:
    """Build both oracle libraries. Returns False when the reference is absent."""
    native = _native(reference if reference is not None else default_reference())
    if not native.is_dir():
        return False
    cuda_home = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
    nvcc = str(cuda_home / "bin" / "nvcc")
    cxx = shutil.which("g++") or "g++"
    obj_dir = OUT_DIR / "obj"
    obj_dir.mkdir(parents=True, exist_ok=True)
    includes = _include_flags(native, cuda_home)
    library = OUT_DIR / "libref_hybridsplat.so"
    prepare_library = OUT_DIR / "libref_prepare.so"

    sources = _sources(native)
    newest_source = max(
        max(p.stat().st_mtime for p, _, _ in sources),
        Path(__file__).stat().st_mtime,
    )
    if (
        not force
        and library.exists()
        and prepare_library.exists()
        and library.stat().st_mtime >= newest_source
    ):
        return True

    jobs_list = []
    objects = []
    for source, language, options in sources:
        target = obj_dir / (source.name + ".o")
        objects.append(target)
        if language == "cuda":
            command = [nvcc, *_RELEASE, *_CUDA_COMMON, *_DEFINES, *includes, *options,
                       "-c", str(source), "-o", str(target)]
        else:
            command = [cxx, *_RELEASE, *_CXX_COMMON, *_DEFINES, *includes, *options,
                       "-c", str(source), "-o", str(target)]
        jobs_list.append((command, target))
    with concurrent.futures.ThreadPoolExecutor(max_workers=jobs) as pool:
        for _ in pool.map(_compile, jobs_list):
            pass

    link = [
        nvcc, "-shared", "-gencode", "arch=compute_100,code=sm_100",
        *[str(o) for o in objects],
        "-o", str(library),
        f"-L{cuda_home / 'lib64'}", "-lcudart", "-lcuda", "-lcublas", "-lcusolver", "-ldl",
    ]
    _compile((link, library))

    # Host-only NPZ activation: g++ on the reference file, same Release flags.
    prepare_obj = obj_dir / "flashgs_prepare_host.o"
    _compile(([cxx, *_RELEASE, *_CXX_COMMON, *_DEFINES, *includes,
               "-c", str(native / "rasterizer" / "flashgs_prepare.cpp"),
               "-o", str(prepare_obj)], prepare_obj))
    _compile(([cxx, "-shared", str(prepare_obj), "-o", str(prepare_library)], prepare_library))
    return True


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference", type=Path, default=None)
    parser.add_argument("--jobs", type=int, default=8)
    parser.add_argument("--force", action="store_true")
    arguments = parser.parse_args()
    built = build(arguments.reference, arguments.jobs, arguments.force)
    print("reference oracle built" if built else "reference checkout absent; nothing built")
    return 0


if __name__ == "__main__":
    sys.exit(main())
