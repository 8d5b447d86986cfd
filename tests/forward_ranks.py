"""Two ranks on two GPUs forward an indexer layer's picks across a stage cut at a shared layer (cuts
0 and 39: layer 39 attends with layer 38's picks) for five calls, with the forwarder
glmkv.dist.picks_forwarder builds there. The receiver checks, in every call, that the picks it
attends with are the sender's picks of the call before, bit for bit. Run by
tests/test_gpu_forward.py under torch.distributed.run."""
import os
import pathlib
import sys

ROOT = pathlib.Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT / "kern-glm53_b200")]

import torch  # noqa: E402

from glmkv import dist as gd  # noqa: E402


def main():
    world, rank, local = gd.env()
    assert world == 2
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    gd.init("nccl", timeout_s=60, device=dev)
    T = 48
    ind = {38: torch.zeros(T, 2048, dtype=torch.int32, device=dev)} if rank == 0 else {}
    tlen = torch.zeros(T, dtype=torch.int32, device=dev)
    fwd = gd.picks_forwarder((0, 39), rank, T, dev, ind=ind, tlen=tlen)
    kind = type(fwd).__name__
    base = torch.arange(T * 2048, dtype=torch.int32, device=dev).view(T, 2048)
    bad = 0
    for c in range(5):
        fwd.begin_call()
        if rank == 1 and c >= 1:  # the picks this call attends with: the sender's of call c - 1
            torch.cuda.synchronize()
            a, t = fwd.received(38)
            bad += int(not torch.equal(a.view(T, 2048), base + 1000 * (c - 1)))
            bad += int(not torch.equal(t, torch.full_like(t, c)))
        if rank == 0:
            fwd.hook("topk", 38, True)
            ind[38].copy_(base + 1000 * c)
            tlen.fill_(c + 1)
            fwd.hook("topk", 38, False)
        if rank == 1:
            fwd.hook("mla_prep", 77, True)
        fwd.end_call()
    fwd.drain()
    torch.cuda.synchronize()
    gd.barrier()
    fwd.close()  # every rank unmaps its peer's buffers before either frees its own
    gd.barrier()
    print(f"forward {'ok' if bad == 0 else 'BAD'} rank {rank} {kind} mismatches {bad}", flush=True)
    gd.finish()
    sys.exit(0 if bad == 0 else 1)


if __name__ == "__main__":
    main()
