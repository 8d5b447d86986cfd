"""The library's launch switches change how kernels are launched, never what they compute: one layer of
the path (tests/switch_case.py) gives the same bytes with programmatic dependent launch off
(GLMKV_PDL=0) and with SMs reserved (GLMKV_RESERVE_SMS), and the persistent grids shrink by the
reserved SMs. Each setting runs in its own process (the library reads them once per process)."""
import json
import os
import pathlib
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = pathlib.Path(__file__).resolve().parent


def _run(env_extra):
    env = {k: v for k, v in os.environ.items() if k not in ("GLMKV_PDL", "GLMKV_RESERVE_SMS")}
    env.update(env_extra)
    out = subprocess.run([sys.executable, str(HERE / "switch_case.py")], env=env, capture_output=True, text=True,
                         timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    return json.loads(out.stdout.strip().splitlines()[-1])


def test_launch_switches_keep_the_results(cuda):
    base = _run({})
    nopdl = _run({"GLMKV_PDL": "0"})
    reserved = _run({"GLMKV_RESERVE_SMS": "8"})
    assert base["faults"] == nopdl["faults"] == reserved["faults"] == 0
    assert nopdl["digest"] == base["digest"], "GLMKV_PDL=0 changed the outputs"
    assert reserved["digest"] == base["digest"], "GLMKV_RESERVE_SMS changed the outputs"
    sms = base["sms"]
    for entry in ("glm_kv_dequant", "glm_idx_gather", "glm_mla_prep_fp8"):
        g0, b0, s0 = base["shapes"][entry]
        g1, b1, s1 = reserved["shapes"][entry]
        per_sm = g0 // sms
        assert g0 == per_sm * sms and g1 == per_sm * (sms - 8), (entry, g0, g1)
        assert (b0, s0) == (b1, s1)
    assert base["shapes"]["glm_mark_rows"][0] == sms and reserved["shapes"]["glm_mark_rows"][0] == sms - 8
