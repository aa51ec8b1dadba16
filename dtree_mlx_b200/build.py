"""Build ``libdtree_b200.so`` in-tree with nvcc for sm_100a.

The library is a plain C-ABI shared object (``include/dtree_b200.h``) loaded
with ctypes; it is compiled from ``dtree_mlx_b200/csrc/*.cu`` with relocatable
device code and linked against the shared CUDA runtime so it shares the
process's runtime (and streams) with PyTorch.

    python -m dtree_mlx_b200.build [--force] [-j N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "libdtree_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-rdc=true",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    f"-I{ROOT / 'include'}",
    f"-I{CSRC}",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libdtree_b200.so")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps(src: Path) -> list[Path]:
    return [src, *CSRC.glob("*.cuh"), ROOT / "include" / "dtree_b200.h"]


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in _deps(src) if d.exists())


def compile_one(src: Path, force: bool, extra: list[str]) -> Path:
    obj = BUILD / (src.stem + ".o")
    if force or _stale(obj, src):
        cmd = [nvcc(), *ARCH, *COMMON, *extra, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    """Compile every kernel source for sm_100a and link the shared library."""
    BUILD.mkdir(exist_ok=True)
    extra = ["-Xptxas", "-v"] if verbose else []
    srcs = sources()
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: compile_one(s, force, extra), srcs))
    if force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [
            nvcc(),
            *ARCH,
            "-shared",
            "-rdc=true",
            "-cudart",
            "shared",
            *[str(o) for o in objs],
            "-o",
            str(tmp),
            "-Xlinker",
            "-rpath,/usr/local/cuda/lib64",
        ]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("-v", action="store_true", help="pass -Xptxas -v (registers / spills)")
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.j, verbose=a.v))


if __name__ == "__main__":
    main()
