"""Build the B200 KV-cache kernels in-tree.

* ``glmkv/libglmkv.so``      -- the C ABI of ``include/glmkv.h`` (host launchers + kernels).
* ``glmkv/glm_glue_b200.cubin`` -- the same kernels as a cubin with the reference's entry names, for a
  kern manifest.

Both for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``); nvcc cross-compiles without a GPU.

    python kern-glm53_b200/glmkv/build.py [--force] [--verbose]
"""
import argparse
import os
import pathlib
import shutil
import subprocess

OUT = pathlib.Path(__file__).resolve().parent
PKG = OUT.parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = OUT / "libglmkv.so"
CUBIN = OUT / "glm_glue_b200.cubin"
NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-O3", "-lineinfo",
         "-I", str(CSRC), "-I", str(ROOT / "include")]


def _sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "glmkv.h"]


def _stale(out):
    return not out.exists() or any(out.stat().st_mtime < s.stat().st_mtime for s in _sources())


def build(force=False, verbose=False):
    """Compile what is stale; returns (library, cubin)."""
    extra = ["-Xptxas", "-v"] if verbose else []
    if force or _stale(LIB):
        tmp = LIB.with_suffix(".so.tmp")
        subprocess.run([NVCC, *FLAGS, *extra, "-shared", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                        "-o", str(tmp), str(CSRC / "glmkv.cu")], check=True)
        os.replace(tmp, LIB)
    if force or _stale(CUBIN):
        tmp = CUBIN.with_suffix(".cubin.tmp")
        subprocess.run([NVCC, *FLAGS, *extra, "-cubin", "-o", str(tmp), str(CSRC / "glm_glue_b200.cu")], check=True)
        os.replace(tmp, CUBIN)
    return LIB, CUBIN


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register / spill / smem usage")
    a = ap.parse_args()
    print(*build(a.force, a.verbose), sep="\n")
