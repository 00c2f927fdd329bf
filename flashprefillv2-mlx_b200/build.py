"""Build ``fpv2/_lib/libfpv2_b200.so`` from ``csrc/*.cu`` with nvcc for sm_100a.

The library is a plain C-ABI shared object (include/fpv2_b200.h) with the CUDA
runtime linked statically; it has no PyTorch dependency. Objects are compiled
in parallel into ``_build/`` and relinked only when a source or header is newer
than the library.

    python flashprefillv2-mlx_b200/build.py [--force] [--verbose] [--debug-bounds]

``--debug-bounds`` builds ``fpv2/_lib/libfpv2_b200_debug.so`` instead (objects in
``_build_debug/``): the same kernels, which also report every block-list entry,
count or page index they had to clamp into range in the device status word
(bit 8, read with ``fpv2_device_status``). Point ``FPV2_LIBRARY`` at it to use it.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
BUILD = HERE / "_build"
BUILD_DEBUG = HERE / "_build_debug"
LIB_DIR = HERE / "fpv2" / "_lib"
LIB = LIB_DIR / "libfpv2_b200.so"
LIB_DEBUG = LIB_DIR / "libfpv2_b200_debug.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    f"-I{INCLUDE}",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def headers() -> list[Path]:
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _compile(src: Path, verbose: bool, extra: list[str], bdir: Path = BUILD) -> Path:
    obj = bdir / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, flush=True)
    return obj


def up_to_date(lib: Path = LIB) -> bool:
    if not lib.exists():
        return False
    t = lib.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in [*sources(), *headers(), Path(__file__)])


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False,
          debug_bounds: bool = False) -> Path:
    """Compile every CUDA source for sm_100a and link the shared library (the
    bounds-reporting debug library with ``debug_bounds``)."""
    lib = LIB_DEBUG if debug_bounds else LIB
    bdir = BUILD_DEBUG if debug_bounds else BUILD
    if not force and not ptxas_info and up_to_date(lib):
        return lib
    bdir.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    if debug_bounds:
        extra.append("-DFPV2_DEBUG_BOUNDS=1")
    workers = min(len(sources()), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=workers) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose or ptxas_info, extra, bdir), sources()))
    tmp = lib.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs),
           "-ldl", "-lpthread", "-lrt"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, lib)
    return lib


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills/smem")
    ap.add_argument("--debug-bounds", action="store_true",
                    help="build libfpv2_b200_debug.so, which reports clamped list entries")
    args = ap.parse_args(argv)
    lib = build(force=args.force, verbose=args.verbose, ptxas_info=args.ptxas_info,
                debug_bounds=args.debug_bounds)
    print(lib)
    return 0


if __name__ == "__main__":
    sys.exit(main())
