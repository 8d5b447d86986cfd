"""The bf16 instruction identities the kernels rely on for bit-exactness, checked exhaustively on the
GPU (``tests/bf16_identities.cu``): packed bf16 add and multiply equal the reference's f32 operation
followed by bf16 rounding, the mixed-precision ``fma.rn.f32.bf16`` equals the f32 FMA of the widened
values, and ``max.xorsign.abs.bf16x2`` gives ``fmaxf(|a|, |b|)``. Over all 2^32 operand pairs."""
import os
import pathlib
import shutil
import subprocess

import pytest

HERE = pathlib.Path(__file__).resolve().parent


@pytest.mark.gpu
def test_bf16_instruction_identities(tmp_path):
    nvcc = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
    exe = tmp_path / "bf16_identities"
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-o", str(exe),
                    str(HERE / "bf16_identities.cu")], check=True)
    p = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    print(p.stdout)
    assert p.returncode == 0, p.stdout + p.stderr
    counts = dict(kv.split("=") for kv in p.stdout.split())
    assert all(v.split("/")[0] == "0" for v in counts.values()), counts
