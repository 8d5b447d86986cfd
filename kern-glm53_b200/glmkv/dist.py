"""Process-per-GPU plumbing for the layer-group stages (torch.distributed; NCCL on GPUs, gloo on CPU).

Each rank owns whole layers, so the cache path itself exchanges nothing while every stage starts at
an indexer layer. A placement that cuts at a shared layer adds one exchange: the picks of the indexer
layer before the cut travel to the stage that starts there (`PicksForwarder`, NCCL send / recv over
NVLink, overlapped with the stage's kernels). The other helpers place the stages and combine timings:
the slowest rank's time is the job's (every rank takes the same collective steps in the same order,
so a rank that fails or leaves makes the others' next collective end with an error after the process
group's timeout instead of hanging).
"""
import datetime
import os

import torch
import torch.distributed as dist

from . import stage


def env():
    """(world, rank, local_rank) from the torchrun environment (1, 0, 0 without it)."""
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init(backend, timeout_s=300, device=None):
    """Join the process group when there is more than one rank; returns (world, rank, local_rank)."""
    world, rank, local = env()
    if world > 1 and not dist.is_initialized():
        kw = {"device_id": device} if device is not None and backend == "nccl" else {}
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return world, rank, local


def assignment(world, **kw):
    """[(first, last)] layer range of every rank: stage cuts balanced by bytes (at indexer layers unless
    `any_layer=True` is passed on to stage.cuts)."""
    c = list(stage.cuts(world, **kw)) + [stage.LAYERS]
    return [(c[i], c[i + 1]) for i in range(world)]


class PicksForwarder:
    """The one exchange of a placement with cuts at shared layers: per call, the picks of indexer layer
    `src` (ind [T, 2048] i32, after the row plan, and tlen [T] i32) go from the rank that owns `src` to
    the rank whose stage starts at a shared layer that attends with them (stage.forwarded_picks).

    Stages form a pipeline: while the receiving stage works on call c, the sending stage works on call
    c + 1. So a call's picks are received one call ahead: `begin_call` makes the stream wait for the
    receive posted at the previous call's start (the picks this call's layers attend with) and posts
    the receive of the next call's, into the other of two buffers. The sender posts its sends once the
    row plan of `src` has rewritten the picks (`hook`, LayerGroup.run_call's on_op); the picks are
    rewritten in place every call, so the next call's row plan of `src` first waits for that send.
    On GPUs sends and receives go on a side stream, so the transfer overlaps the stages' kernels.
    `drain` waits for whatever is still in flight. Every rank posts the same messages in the same order
    each call (ind, then tlen)."""

    def __init__(self, cut_list, rank, T, device, ind=None, tlen=None):
        plan = stage.forwarded_picks(cut_list)
        self.sends = [(dst, src) for snd, dst, src in plan if snd == rank]
        self.recvs = [(snd, src) for snd, dst, src in plan if dst == rank]
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        self.stream = torch.cuda.Stream(self.device) if self.cuda and (self.sends or self.recvs) else None
        self.ind, self.tlen = ind, tlen
        i32 = lambda n: torch.empty(n, dtype=torch.int32, device=self.device)
        self.recv_buf = {src: [(i32(T * 2048), i32(T)) for _ in range(2)] for _, src in self.recvs}
        self.tlen_sent = {src: i32(T) for _, src in self.sends}
        self.pending_send, self.pending_recv = {}, []
        self.calls = 0  # calls begun: the receive posted by call c fills buffer c % 2
        self.done = 0  # the buffer of the last completed receive
        self.bytes_per_call = stage.picks_bytes(T) * (len(self.sends) + len(self.recvs))

    @property
    def active(self):
        return bool(self.sends or self.recvs)

    def _side(self):
        return torch.cuda.stream(self.stream) if self.stream is not None else _null()

    def begin_call(self):
        if self.pending_recv:  # the picks this call's layers attend with
            for w in self.pending_recv:
                w.wait()
            self.pending_recv = []
            self.done = (self.calls - 1) % 2
        if self.stream is not None and self.recvs:  # the buffer about to be refilled was read two calls ago
            self.stream.wait_stream(torch.cuda.current_stream(self.device))
        for snd, src in self.recvs:
            ind, tl = self.recv_buf[src][self.calls % 2]
            with self._side():
                self.pending_recv += [dist.irecv(ind, snd), dist.irecv(tl, snd)]
        self.calls += 1

    def hook(self, op, l, before):
        if op != "topk":
            return
        for dst, src in self.sends:
            if l != src:
                continue
            if before:  # the row plan rewrites these picks: the previous call's send must have read them
                for w in self.pending_send.pop(src, []):
                    w.wait()
                continue
            self.tlen_sent[src].copy_(self.tlen)
            if self.stream is not None:
                self.stream.wait_stream(torch.cuda.current_stream(self.device))
            with self._side():
                self.pending_send[src] = [dist.isend(self.ind[src].view(-1), dst),
                                          dist.isend(self.tlen_sent[src], dst)]

    def end_call(self):
        """Nothing to wait for: the next call's picks are received while this stage works."""

    def drain(self):
        for ws in self.pending_send.values():
            for w in ws:
                w.wait()
        self.pending_send = {}
        if self.pending_recv:
            for w in self.pending_recv:
                w.wait()
            self.pending_recv = []
            self.done = (self.calls - 1) % 2

    def received(self, src):
        """(ind, tlen) of indexer layer `src` of the last completed receive: while a call runs, the picks
        that call attends with; after `drain`, the last call's."""
        return self.recv_buf[src][self.done]


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


def max_over_ranks(value, device=None):
    """The largest `value` over all ranks (the value itself with one rank)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return value
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value, device=None):
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return value
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def gather_objects(obj):
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return [obj]
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, obj)
    return out


def barrier():
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()


def finish():
    if dist.is_initialized():
        dist.destroy_process_group()
