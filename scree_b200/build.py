"""Build libscree_b200.so (all CUDA sources of scree_b200/csrc) for sm_100a.

Usage: ``python -m scree_b200.build`` (or ``build()`` from Python).  Objects go to
``_build/`` at the repository root, the shared library next to this file so it
ships with the package tree.  nvcc cross-compiles, so no GPU is needed.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
ROOT = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = ROOT / "_build"
LIB_PATH = PKG_DIR / "libscree_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-I",
    str(ROOT / "include"),
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _needs_rebuild(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src, *CSRC.glob("*.cuh"), ROOT / "include" / "scree_b200.h"]
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False, force: bool = False) -> Path:
    """Compile every .cu under csrc/ and link libscree_b200.so.  Returns its path."""
    nvcc = _nvcc()
    BUILD_DIR.mkdir(exist_ok=True)
    srcs = _sources()
    objs = [BUILD_DIR / (s.stem + ".o") for s in srcs]

    def compile_one(pair):
        src, obj = pair
        if not force and not ptxas_info and not _needs_rebuild(obj, src):
            return ""
        cmd = [nvcc, *ARCH_FLAGS, *CFLAGS, "-c", str(src), "-o", str(obj)]
        if ptxas_info:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
        return r.stderr if (verbose or ptxas_info) else ""

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for msg in ex.map(compile_one, zip(srcs, objs)):
            if msg:
                print(msg, file=sys.stderr)

    if force or not LIB_PATH.exists() or any(o.stat().st_mtime > LIB_PATH.stat().st_mtime for o in objs):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    p = build(verbose="-v" in sys.argv, ptxas_info="--ptxas" in sys.argv, force="--force" in sys.argv)
    print(p)
