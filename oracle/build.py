"""Build recipe for the test oracles (test infrastructure only).

* ``oracle/_build/libglmoracle.so``: the C restatement in ``glm_oracle.c`` (gcc, OpenMP,
  ``-ffp-contract=off`` so every f32 rounding is the one written in the source).
* ``oracle/_ref/libglmref.so``: the reference's own ``source/glm_glue.cu``, compiled unmodified from
  the reference tree for sm_100a with the host launchers in ``ref_launch.cu``. Built only where the
  reference tree is present; the built library travels with the repository snapshot to the GPU box.

    python oracle/build.py [--ref-root PATH]
"""
import argparse
import os
import pathlib
import shutil
import subprocess

HERE = pathlib.Path(__file__).resolve().parent
BUILD = HERE / "_build"
REF_OUT = HERE / "_ref"
ORACLE_SO = BUILD / "libglmoracle.so"
REF_SO = REF_OUT / "libglmref.so"
DEFAULT_REF_ROOT = pathlib.Path(os.environ.get("GLMKV_REFERENCE_ROOT", "/root/reference"))
NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _run(cmd):
    subprocess.run(cmd, check=True)


def _stale(out, srcs):
    return not out.exists() or any(out.stat().st_mtime < pathlib.Path(s).stat().st_mtime for s in srcs)


def build_oracle(force=False):
    src = HERE / "glm_oracle.c"
    if force or _stale(ORACLE_SO, [src]):
        BUILD.mkdir(exist_ok=True)
        tmp = ORACLE_SO.with_suffix(".so.tmp")
        _run(["gcc", "-O2", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", "-std=c11",
              "-o", str(tmp), str(src), "-lm"])
        os.replace(tmp, ORACLE_SO)
    return ORACLE_SO


def build_ref(ref_root=DEFAULT_REF_ROOT, force=False):
    """Compile the reference glue kernels from the reference tree; returns None when it is absent."""
    glue = pathlib.Path(ref_root) / "source" / "glm_glue.cu"
    if not glue.exists():
        return None
    launch = HERE / "ref_launch.cu"
    if force or _stale(REF_SO, [glue, launch]):
        REF_OUT.mkdir(exist_ok=True)
        tmp = REF_SO.with_suffix(".so.tmp")
        # The reference's own flags for this module (kernels.toml [flags].plain: -std=c++17 -O3).
        _run([NVCC, *GENCODE, "-std=c++17", "-O3", "-lineinfo", "-shared", "-Xcompiler", "-fPIC,-fvisibility=hidden",
              "-I", str(glue.parent), "-o", str(tmp), str(launch)])
        os.replace(tmp, REF_SO)
    return REF_SO


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-root", default=str(DEFAULT_REF_ROOT))
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build_oracle(a.force))
    print(build_ref(a.ref_root, a.force))


if __name__ == "__main__":
    main()
