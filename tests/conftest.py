import os
import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
PKG = ROOT / "kern-glm53_b200"
for p in (str(ROOT), str(PKG), str(ROOT / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long CPU test")


@pytest.fixture(scope="session")
def built_lib():
    """libglmkv.so, (re)built in-tree when stale (nvcc cross-compiles; no GPU needed)."""
    from glmkv import build as pkg_build

    lib, _ = pkg_build.build()
    return lib


@pytest.fixture(scope="session")
def cuda(built_lib):
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    torch.cuda.init()
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def ref(cuda):
    """The reference's own glue kernels (oracle/_ref/libglmref.so), the bit-exact oracle of every GPU
    parity test. A GPU run without them fails: the bit-exact half of the suite must not turn into
    skips or looser oracle checks."""
    from oracle import ref as ref_mod

    if not ref_mod.available():
        pytest.fail("oracle/_ref/libglmref.so is missing: build it with `python oracle/build.py --ref-root "
                    "<kern-glm53 checkout>` where the reference tree is present; it travels with the repository")
    ref_mod.lib()
    return ref_mod
