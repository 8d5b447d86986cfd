"""The tensor-core ceiling of glm_mqa_logits_paged (``tests/tcgen05_rate.cu``): back-to-back
tcgen05.mma from shared memory in the kernel's own operand layout and instruction descriptor, with no
copies and no epilogue, in e4m3 and in bf16.

The e4m3 kind must run at about twice the bf16 rate per SM clock (the dense fp8 rate of the part):
that checks that the MQA's descriptor selects the full-rate fp8 path. The printed rates are the
ceiling the MQA's TFLOP/s is read against."""
import os
import pathlib
import shutil
import subprocess

import pytest

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent


@pytest.mark.gpu
def test_tcgen05_fp8_runs_at_twice_the_bf16_rate(tmp_path):
    nvcc = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
    exe = tmp_path / "tcgen05_rate"
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                    "-I", str(ROOT / "kern-glm53_b200" / "csrc"), "-I", str(ROOT / "include"),
                    "-o", str(exe), str(HERE / "tcgen05_rate.cu"), "-lcuda"], check=True)
    p = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    print(p.stdout)
    assert p.returncode == 0, p.stdout + p.stderr
    # per SM clock (the power cap lowers the clock under a long tensor load): TFLOP/s per MHz
    rate = {ln.split()[0]: float(ln.split()[1]) / float(ln.split()[3]) for ln in p.stdout.splitlines() if "TFLOP/s" in ln}
    assert rate["f8f6f4_e4m3_m128n256"] > 1.8 * rate["f16_bf16_m128n256"], rate
