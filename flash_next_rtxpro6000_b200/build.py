"""Build the sm_100a shared library ``_fnx.so`` in-tree with nvcc.

    python -m flash_next_rtxpro6000_b200.build [--force]

Each ``csrc/*.cu`` file is compiled to an object in parallel, then linked into one
shared library with the CUDA runtime linked statically (the library then depends only on
the driver, not on a particular libcudart).
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB_PATH = PKG / "_fnx.so"
OBJ_DIR = PKG / "_build"

SOURCES = ["fnx_api.cu", "dense_gemv.cu", "dense_gemv_slice.cu", "dense_gemv_norm.cu", "dense_tc.cu",
           "moe_gemv.cu",
           "moe_fused.cu", "moe_lean.cu", "nvfp4_codec.cu", "router.cu", "topk1.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-I" + str(INCLUDE)]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the sm_100a library cannot be built")
    return cand


def _inputs():
    return [CSRC / s for s in SOURCES] + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + \
        sorted(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    t = LIB_PATH.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _inputs())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if any source is newer than it; returns its path."""
    if not force and up_to_date():
        return LIB_PATH
    OBJ_DIR.mkdir(exist_ok=True)
    cc = nvcc()
    extra = ["-Xptxas", "-v"] if verbose else []

    def compile_one(src: str) -> Path:
        obj = OBJ_DIR / (Path(src).stem + ".o")
        cmd = [cc, *ARCH, *FLAGS, *extra, "-c", str(CSRC / src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        if verbose:
            sys.stderr.write(r.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(compile_one, SOURCES))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [cc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
