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
