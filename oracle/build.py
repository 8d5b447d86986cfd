"""Build recipe for the test oracles (test infrastructure only).

* ``oracle/_build/libglmoracle.so``: the C restatement in ``glm_oracle.c`` (gcc, OpenMP,
  ``-ffp-contract=off`` so every f32 rounding is the one written in the source).
* ``oracle/_ref/libglmref.so``: the reference's own ``source/glm_glue.cu``, compiled unmodified from
  the reference tree for sm_100a with the host launchers in ``ref_launch.cu``. Built only where the
  reference tree is given (``--ref-root`` or ``GLMKV_REFERENCE_ROOT``); the built library travels with
  the repository snapshot to the GPU box.

    python oracle/build.py --ref-root path/to/kern-glm53
    GLMKV_REFERENCE_ROOT=path/to/kern-glm53 python oracle/build.py
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
ENV_REF_ROOT = "GLMKV_REFERENCE_ROOT"
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


def reference_root(ref_root=None):
    """The kern-glm53 checkout: the argument, else GLMKV_REFERENCE_ROOT; None when neither is given."""
    root = ref_root or os.environ.get(ENV_REF_ROOT)
    return pathlib.Path(root) if root else None


def build_ref(ref_root=None, force=False):
    """Compile the reference glue kernels from the reference tree (the argument, else
    GLMKV_REFERENCE_ROOT). Returns None when no tree is given; raises when the one given has no
    source/glm_glue.cu."""
    root = reference_root(ref_root)
    if root is None:
        return None
    glue = root / "source" / "glm_glue.cu"
    if not glue.exists():
        raise FileNotFoundError(f"{root} has no source/glm_glue.cu: not a kern-glm53 checkout")
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
    ap.add_argument("--ref-root", default=None, help=f"the kern-glm53 checkout (default: ${ENV_REF_ROOT})")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build_oracle(a.force))
    if reference_root(a.ref_root) is None:
        raise SystemExit(f"the reference glue kernels need the kern-glm53 checkout: --ref-root or ${ENV_REF_ROOT}")
    print(build_ref(a.ref_root, a.force))


if __name__ == "__main__":
    main()
