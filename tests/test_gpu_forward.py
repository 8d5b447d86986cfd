"""The picks' exchange of a placement with a stage cut at a shared layer, on two GPUs: two ranks run
tests/forward_ranks.py, and the receiving rank gets, call by call, exactly the picks the sending rank
made one call before. Needs two GPUs (skipped on a one-GPU box); the host logic of the same exchange
is tested on CPU with gloo ranks in tests/test_stage.py."""
import os
import pathlib
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

HERE = pathlib.Path(__file__).resolve().parent


def test_picks_forwarded_across_a_cut_at_a_shared_layer(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES=os.environ.get("CUDA_VISIBLE_DEVICES", "0,1"))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", "29531", str(HERE / "forward_ranks.py")]
    p = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env=env)
    out = p.stdout + p.stderr
    assert p.returncode == 0, out[-3000:]
    assert "forward ok rank 1 PeerCopyForwarder mismatches 0" in out, out[-3000:]
    assert "forward ok rank 0 PeerCopyForwarder" in out, out[-3000:]
