"""Build the in-tree CUDA shared library ``libpolarpack_b200.so`` for sm_100a.

    python -m polar_pack_b200.build [--verbose]

Compiles every ``csrc/*.cu`` with nvcc (``-gencode arch=compute_100a,
code=sm_100a``), links them with the static CUDA runtime into one shared
object next to this file, and skips the work when the library is newer
than all sources.  nvcc cross-compiles, so no GPU is needed.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB_NAME = "libpolarpack_b200.so"
LIB_PATH = PKG / LIB_NAME
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2,-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-Xptxas", "-v", "-I", str(INCLUDE)]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def deps() -> list[Path]:
    return sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    t = LIB_PATH.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in deps())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB_PATH
    nvcc = nvcc_path()
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    objs = []
    log = []

    def compile_one(src: Path):
        obj = objdir / (src.stem + ".o")
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, obj, cmd, r

    # the translation units are independent: compile them in parallel
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(sources()), os.cpu_count() or 1))) as pool:
        results = list(pool.map(compile_one, sources()))
    for src, obj, cmd, r in results:
        log.append(f"$ {' '.join(cmd)}\n{r.stdout}{r.stderr}")
        if r.returncode != 0:
            sys.stderr.write("\n".join(log))
            raise RuntimeError(f"nvcc failed on {src.name}")
        objs.append(str(obj))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    log.append(f"$ {' '.join(cmd)}\n{r.stdout}{r.stderr}")
    if r.returncode != 0:
        sys.stderr.write("\n".join(log))
        raise RuntimeError("link failed")
    os.replace(tmp, LIB_PATH)
    (objdir / "build.log").write_text("\n".join(log))
    if verbose:
        print("\n".join(log))
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
