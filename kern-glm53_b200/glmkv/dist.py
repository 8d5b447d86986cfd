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
    c + 1. So a call's picks are received one call ahead, into alternating buffers: the receive posted
    during call c is waited for when call c + 1 begins (`begin_call`), and those are the picks call
    c + 1's layers attend with. The sender posts its sends once the row plan of `src` has rewritten the
    picks (`hook`, LayerGroup.run_call's on_op); the picks are rewritten in place every call, so the
    next call's row plan of `src` first waits for that send.

    The receiver posts its receive when it reaches the layer at the same place in its stage as `src` in
    the sender's (or at the call's end, `end_call`, if no such layer runs), not at the call's start: a
    transfer kernel waits on its SMs until the peer's half is posted, and one posted at the call's start
    sat there for most of the call, beside the stage's persistent kernels (0.33 ms a call at 8 GPUs).
    On GPUs sends and receives go on a side stream, so the transfer overlaps the stages' kernels.
    `drain` waits for whatever is still in flight. Every rank posts the same messages in the same order
    each call (ind, then tlen)."""

    def __init__(self, cut_list, rank, T, device, ind=None, tlen=None):
        plan = stage.forwarded_picks(cut_list)
        c = list(cut_list) + [stage.LAYERS]
        self.sends = [(dst, src) for snd, dst, src in plan if snd == rank]
        # (sender, source layer, the layer of this stage at which the receive is posted)
        self.recvs = [(snd, src, min(c[rank] + (src - c[snd]), c[rank + 1] - 1)) for snd, dst, src in plan
                      if dst == rank]
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        self.stream = torch.cuda.Stream(self.device) if self.cuda and (self.sends or self.recvs) else None
        self.ind, self.tlen = ind, tlen
        i32 = lambda n: torch.empty(n, dtype=torch.int32, device=self.device)
        self.recv_buf = {src: [(i32(T * 2048), i32(T)) for _ in range(2)] for _, src, _ in self.recvs}
        self.tlen_sent = {src: i32(T) for _, src in self.sends}
        self.pending_send, self.pending_recv = {}, []
        self.posted = set()  # sources whose receive this call has posted
        self.calls = 0  # calls begun: the receive posted during call c (0-based) fills buffer c % 2
        self.done = 0  # the buffer of the last completed receive
        self.bytes_per_call = stage.picks_bytes(T) * (len(self.sends) + len(self.recvs))

    @property
    def active(self):
        return bool(self.sends or self.recvs)

    def _side(self):
        return torch.cuda.stream(self.stream) if self.stream is not None else _null()

    def _wait_recvs(self):
        if self.pending_recv:
            for w in self.pending_recv:
                w.wait()
            self.pending_recv = []
            self.done = (self.calls - 1) % 2

    def _post_recv(self, snd, src):
        if self.stream is not None:  # the buffer about to be refilled was read two calls ago
            self.stream.wait_stream(torch.cuda.current_stream(self.device))
        ind, tl = self.recv_buf[src][(self.calls - 1) % 2]
        with self._side():
            self.pending_recv += [dist.irecv(ind, snd), dist.irecv(tl, snd)]
        self.posted.add(src)

    def begin_call(self):
        self._wait_recvs()  # the picks this call's layers attend with
        self.calls += 1
        self.posted = set()

    def hook(self, op, l, before):
        if op == "mla_prep" and before:
            for snd, src, at in self.recvs:
                if l == at and src not in self.posted:
                    self._post_recv(snd, src)
            return
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
        """Posts the receives this call has not posted yet (their layer did not run)."""
        for snd, src, _ in self.recvs:
            if src not in self.posted:
                self._post_recv(snd, src)

    def drain(self):
        for ws in self.pending_send.values():
            for w in ws:
                w.wait()
        self.pending_send = {}
        self._wait_recvs()

    def close(self):
        """Nothing to unmap: the process group owns the transfers."""

    def received(self, src):
        """(ind, tlen) of indexer layer `src` of the last completed receive: while a call runs, the picks
        that call attends with; after `drain`, the last call's."""
        return self.recv_buf[src][self.done]


class PeerCopyForwarder:
    """The same exchange as PicksForwarder, moved by the copy engines instead of NCCL's kernels, so no
    SM of either GPU waits on it.

    The receiver exports its two buffer sets (ind [T, 2048] i32 and tlen [T] i32) and a flag word to the
    sender through CUDA IPC; the sender exports a flag word back. For call i the sender's side stream,
    after the row plan of `src`:
      1. waits (a stream memory operation, no kernel) until its own flag reads i - 1: the receiver has
         finished call i - 1, the last one that attended with the picks in buffer i % 2;
      2. copies the picks into the receiver's buffer i % 2 (cudaMemcpyAsync across NVLink);
      3. writes i + 1 into the receiver's flag (a stream write, after the copies complete).
    The receiver's stream waits for its flag to read i when call i begins (the previous call's picks
    have landed, received one call ahead as in PicksForwarder), and writes i into the sender's flag
    when call i ends. The next call's row plan of `src` waits for the copy of this call's picks. No
    wait depends on one that follows it, so the two GPUs cannot deadlock. Built by `picks_forwarder`
    when every rank can use it."""

    def __init__(self, cut_list, rank, T, device, ind, tlen, exports):
        from cuda.bindings import driver as cu, runtime as rt

        self.cu, self.rt = cu, rt
        plan = stage.forwarded_picks(cut_list)
        self.sends = [(dst, src) for snd, dst, src in plan if snd == rank]
        self.recvs = [(snd, src) for snd, dst, src in plan if dst == rank]
        self.device = torch.device(device)
        self.ind, self.tlen = ind, tlen
        self.stream = torch.cuda.Stream(self.device)
        self.bytes_per_call = stage.picks_bytes(T) * (len(self.sends) + len(self.recvs))
        self.T, self.calls = T, 0
        loc = exports[rank]
        self.recv_buf = {src: loc["bufs"][src] for _, src in self.recvs}  # local tensors
        self.flag = loc["flag"]  # this rank's flag words: [0] the receive flag, [1] the send flag
        self._opened = {}
        # the peers' memory: for a send, the receiver's buffers and receive flag; for a receive, the
        # sender's send flag
        self.peer = {}
        for dst, src in self.sends:
            pe = exports[dst]["ipc"]
            self.peer[("send", src)] = {"bufs": [(self._open(a), self._open(b)) for a, b in pe["bufs"][src]],
                                        "flag": self._open(pe["flag"]) + 0}
        for snd, src in self.recvs:
            self.peer[("recv", src)] = {"flag": self._open(exports[snd]["ipc"]["flag"]) + 4}
        self.tlen_sent = {src: torch.empty(T, dtype=torch.int32, device=self.device) for _, src in self.sends}
        self.copied = {src: torch.cuda.Event() for _, src in self.sends}
        self.copy_pending = set()

    # ---- CUDA IPC and stream memory operations
    def _ck(self, r, what):
        err = r[0]
        if int(err) != 0:
            raise RuntimeError(f"{what}: {err}")
        return r[1] if len(r) == 2 else r[1:]

    def _open(self, exp):
        handle, off = exp
        if handle not in self._opened:
            h = self.rt.cudaIpcMemHandle_t()
            h.reserved = handle
            self._opened[handle] = int(self._ck(self.rt.cudaIpcOpenMemHandle(h, self.rt.cudaIpcMemLazyEnablePeerAccess),
                                                "cudaIpcOpenMemHandle"))
        return self._opened[handle] + off

    def _wait(self, stream, addr, value):
        self._ck(self.cu.cuStreamWaitValue32(self.cu.CUstream(stream.cuda_stream), self.cu.CUdeviceptr(addr),
                                             value & 0xffffffff,
                                             self.cu.CUstreamWaitValue_flags.CU_STREAM_WAIT_VALUE_GEQ),
                 "cuStreamWaitValue32")

    def _write(self, stream, addr, value):
        self._ck(self.cu.cuStreamWriteValue32(self.cu.CUstream(stream.cuda_stream), self.cu.CUdeviceptr(addr),
                                              value & 0xffffffff,
                                              self.cu.CUstreamWriteValue_flags.CU_STREAM_WRITE_VALUE_DEFAULT),
                 "cuStreamWriteValue32")

    def _copy(self, dst, src_ptr, nbytes):
        self._ck(self.rt.cudaMemcpyAsync(dst, src_ptr, nbytes, self.rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice,
                                         self.rt.cudaStream_t(self.stream.cuda_stream)), "cudaMemcpyAsync")

    # ---- the forwarder's interface (as PicksForwarder)
    @property
    def active(self):
        return bool(self.sends or self.recvs)

    def begin_call(self):
        i = self.calls
        main = torch.cuda.current_stream(self.device)
        if self.recvs and i >= 1:  # the previous call's picks have landed
            self._wait(main, self.flag.data_ptr(), i)
        self.calls += 1

    def hook(self, op, l, before):
        if op != "topk":
            return
        i = self.calls - 1
        main = torch.cuda.current_stream(self.device)
        for dst, src in self.sends:
            if l != src:
                continue
            if before:  # the row plan rewrites these picks: the previous call's copy must have read them
                if src in self.copy_pending:
                    main.wait_event(self.copied[src])
                continue
            self.tlen_sent[src].copy_(self.tlen)
            self.stream.wait_stream(main)
            pe = self.peer[("send", src)]
            if i >= 2:  # the receiver is done with buffer i % 2 (it attended with it in call i - 1)
                self._wait(self.stream, self.flag.data_ptr() + 4, i - 1)
            dind, dtl = pe["bufs"][i % 2]
            self._copy(dind, self.ind[src].data_ptr(), self.T * 2048 * 4)
            self._copy(dtl, self.tlen_sent[src].data_ptr(), self.T * 4)
            self._write(self.stream, pe["flag"], i + 1)
            self.copied[src].record(self.stream)
            self.copy_pending.add(src)

    def end_call(self):
        i = self.calls - 1
        if self.recvs and i >= 1:  # done attending with the picks of call i - 1: their buffer is free
            main = torch.cuda.current_stream(self.device)
            for snd, src in self.recvs:
                self._write(main, self.peer[("recv", src)]["flag"], i)

    def drain(self):
        main = torch.cuda.current_stream(self.device)
        for src in self.copy_pending:
            main.wait_event(self.copied[src])

    def close(self):
        """Unmaps the peers' buffers once this rank's copies and stream operations have completed. Every
        rank closes before any rank frees the buffers it exported (they live as long as the process):
        callers put a barrier after it, as `picks_forwarder` puts one before the first call."""
        self.drain()
        torch.cuda.current_stream(self.device).wait_stream(self.stream)
        torch.cuda.synchronize(self.device)
        for base in self._opened.values():
            self._ck(self.rt.cudaIpcCloseMemHandle(base), "cudaIpcCloseMemHandle")
        self._opened.clear()
        self.peer.clear()
        self.sends, self.recvs = [], []

    def received(self, src):
        """(ind, tlen) of indexer layer `src` that the current (or, between calls, the last) call
        attends with."""
        return self.recv_buf[src][(self.calls - 2) % 2]


def _ipc_export(t):
    """(IPC handle bytes of t's allocation, t's offset in it)."""
    from cuda.bindings import driver as cu, runtime as rt

    err, base, _ = cu.cuMemGetAddressRange(cu.CUdeviceptr(t.data_ptr()))
    if int(err) != 0:
        raise RuntimeError(f"cuMemGetAddressRange: {err}")
    err, h = rt.cudaIpcGetMemHandle(int(base))
    if int(err) != 0:
        raise RuntimeError(f"cudaIpcGetMemHandle: {err}")
    return bytes(h.reserved), t.data_ptr() - int(base)


def picks_forwarder(cut_list, rank, T, device, ind=None, tlen=None):
    """The forwarder of the picks for this rank: PeerCopyForwarder (copy engines, CUDA IPC, stream
    memory operations) on GPUs when every rank can set it up, else PicksForwarder (NCCL or gloo
    send/recv). A collective: every rank calls it, with the same cuts."""
    device = torch.device(device)
    plan = stage.forwarded_picks(cut_list)
    if device.type != "cuda" or not plan or not dist.is_initialized():
        return PicksForwarder(cut_list, rank, T, device, ind=ind, tlen=tlen)
    ok, local = True, {"bufs": {}}
    try:
        from cuda.bindings import driver as cu  # noqa: F401

        i32 = lambda n: torch.zeros(n, dtype=torch.int32, device=device)
        flag = i32(64)  # its own allocation: [0] the receive flag, [1] the send flag
        bufs = {src: [(i32(T * 2048), i32(T)) for _ in range(2)] for snd, dst, src in plan if dst == rank}
        local = {"bufs": bufs, "flag": flag}
        ipc = {"flag": _ipc_export(flag), "bufs": {src: [(_ipc_export(a), _ipc_export(b)) for a, b in v]
                                                   for src, v in bufs.items()}}
        torch.cuda.synchronize(device)
    except Exception:  # noqa: BLE001 - no IPC here: every rank falls back together
        ok, ipc = False, None
    everyone = gather_objects({"ok": ok, "ipc": ipc})
    if not all(e["ok"] for e in everyone):
        return PicksForwarder(cut_list, rank, T, device, ind=ind, tlen=tlen)
    exports = [{**e, **(local if r == rank else {})} for r, e in enumerate(everyone)]
    fwd = PeerCopyForwarder(cut_list, rank, T, device, ind, tlen, exports)
    torch.cuda.synchronize(device)
    barrier()  # every flag is zero and every peer mapping open before the first call
    return fwd


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
