"""Build ``fpv2/_lib/libfpv2_b200.so`` from ``csrc/*.cu`` with nvcc for sm_100a.

The library is a plain C-ABI shared object (include/fpv2_b200.h) with the CUDA
runtime linked statically; it has no PyTorch dependency. Objects are compiled
in parallel into ``_build/`` and relinked only when a source or header is newer
than the library.

    python flashprefillv2-mlx_b200/build.py [--force] [--verbose]
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
LIB_DIR = HERE / "fpv2" / "_lib"
LIB = LIB_DIR / "libfpv2_b200.so"

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


def _compile(src: Path, verbose: bool, extra: list[str]) -> Path:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, flush=True)
    return obj


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in [*sources(), *headers(), Path(__file__)])


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile every CUDA source for sm_100a and link the shared library."""
    if not force and not ptxas_info and up_to_date():
        return LIB
    BUILD.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    workers = min(len(sources()), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=workers) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose or ptxas_info, extra), sources()))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs),
           "-ldl", "-lpthread", "-lrt"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills/smem")
    args = ap.parse_args(argv)
    lib = build(force=args.force, verbose=args.verbose, ptxas_info=args.ptxas_info)
    print(lib)
    return 0


if __name__ == "__main__":
    sys.exit(main())
