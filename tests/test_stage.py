"""Host logic of the layer-group stages: cuts, the byte model, and the multi-process plumbing (gloo,
two ranks on CPU), including a rank that fails: the survivor's next collective ends with an error."""
import multiprocessing as mp
import os
import socket

import pytest

from glmkv import stage, traffic


def test_cuts_are_indexer_layers_and_cover_the_model():
    for n in range(1, 22):
        c = stage.cuts(n)
        assert len(c) == n and c[0] == 0 and list(c) == sorted(set(c))
        assert set(c) <= stage.FULL
    assert stage.cuts(2) == (0, 38)
    assert stage.cuts(4) == (0, 18, 38, 58)  # the reference's own deployment (README.md:13-16)
    with pytest.raises(ValueError):
        stage.cuts(22)


def test_eight_stage_balance_is_the_indexer_layer_bound():
    c = list(stage.cuts(8)) + [78]
    cost = [sum(stage.layer_bytes(l, 16384, 1 << 20) for l in range(c[i], c[i + 1])) for i in range(8)]
    total = sum(stage.layer_bytes(l, 16384, 1 << 20) for l in range(78))
    # 19 blocks of 4 layers after layers 0 and 1: no split of 8 can hold fewer than 3 blocks in a stage
    assert max(c[i + 1] - c[i] for i in range(8)) == 12
    assert total / max(cost) == pytest.approx(6.53, abs=0.01)


def test_any_layer_cuts_and_forwarded_picks():
    T, ctx = 16384, 548864
    total = sum(stage.layer_bytes(l, T, ctx) for l in range(78))
    # where the exchange does not pay for itself the solver keeps to indexer layers (2 and 4 stages: the
    # reference's own cuts at 4)
    for n, want in ((2, (0, 38)), (4, (0, 18, 38, 58)), (8, (0, 9, 18, 28, 38, 48, 58, 68))):
        c = stage.cuts(n, T=T, ctx=ctx, any_layer=True)
        assert c == want
    c8 = stage.cuts(8, T=T, ctx=ctx, any_layer=True)
    cc = list(c8) + [78]
    cost = [sum(stage.layer_bytes(l, T, ctx) for l in range(cc[i], cc[i + 1])) for i in range(8)]
    assert total / max(cost) > 7.4  # against 6.54 with cuts at indexer layers only
    # stages starting at shared layers 9, 28, 48, 68 attend with the picks of layers 6, 26, 46, 66
    assert stage.forwarded_picks(c8) == [(0, 1, 6), (2, 3, 26), (4, 5, 46), (6, 7, 66)]
    assert stage.forwarded_picks((0, 9, 18)) == [(0, 1, 6)]
    assert stage.forwarded_picks(stage.cuts(4)) == []
    assert [stage.picks_source(l) for l in (0, 2, 3, 5, 6, 9, 77)] == [0, 2, 2, 2, 6, 6, 74]


def test_traffic_model():
    assert traffic.kv_dequant(1) == 1808 and traffic.idx_gather(1) == 264 and traffic.topk(1) == 16396
    assert traffic.mla_prep(1, True, "fp8") == 8496
    assert traffic.mla_prep(1, False, "fp8") == 8108
    assert traffic.mla_prep(1, True, "bf16") - traffic.mla_prep(1, True, "fp8") == 496
    assert traffic.layer(16384, 1 << 20, True) == 8496 * 16384 + 264 * (1 << 20) + 16396 * 16384 + 1808 * (1 << 20)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, q, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    from glmkv import dist as gd

    try:
        gd.init("gloo", timeout_s=10)
        mine = gd.assignment(world)[rank]
        ranges = gd.gather_objects(mine)
        slowest = gd.max_over_ranks(1.0 + rank)
        launches = gd.sum_over_ranks(10 * (rank + 1))
        if rank == fail_rank:
            os._exit(3)  # leaves between steps, before the next collective
        gd.barrier()
        gd.finish()
        q.put((rank, "ok", ranges, slowest, launches))
    except Exception as e:  # noqa: BLE001 - the survivor reports what ended its collective
        q.put((rank, "error", type(e).__name__, str(e)[:200], None))
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank_main, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in ps:
        p.start()
    out = []
    for p in ps:
        p.join(timeout=120)
        assert not p.is_alive(), "a rank hung"
    while not q.empty():
        out.append(q.get())
    return sorted(out, key=lambda x: x[0]), [p.exitcode for p in ps]


def test_two_ranks_place_stages_and_combine_timings():
    res, codes = _run(2)
    assert codes == [0, 0]
    for rank, status, ranges, slowest, launches in res:
        assert status == "ok"
        assert ranges == [(0, 38), (38, 78)]
        assert slowest == 2.0 and launches == 30.0


def test_a_rank_that_leaves_is_detected_not_waited_for():
    res, codes = _run(2, fail_rank=1)
    assert codes[1] == 3
    assert len(res) == 1 and res[0][0] == 0 and res[0][1] == "error"


def _forward_main(rank, world, port, q, calls):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    import torch
    import torch.distributed as dist
    from glmkv import dist as gd

    try:
        gd.init("gloo", timeout_s=20)
        T = 16
        cuts = (0, 39)  # layer 39 attends with layer 38's picks, which rank 0 owns
        ind = {38: torch.zeros(T, 2048, dtype=torch.int32)} if rank == 0 else {}
        tlen = torch.zeros(T, dtype=torch.int32)
        fwd = gd.PicksForwarder(cuts, rank, T, "cpu", ind=ind, tlen=tlen)
        got = []
        for c in range(calls):
            fwd.begin_call()
            if rank == 1 and c > 0:  # this call attends with the picks the sender made one call earlier
                a, t = fwd.received(38)
                got.append((int(a[0]), int(a[-1]), int(t[0])))
            if rank == 0:  # the row plan of layer 38 rewrites its picks and tlen, then they are sent
                fwd.hook("topk", 38, True)
                ind[38].copy_(torch.arange(T * 2048, dtype=torch.int32).view(T, 2048) + 1000 * c)
                tlen.fill_(c + 1)
                fwd.hook("topk", 38, False)
            if rank == 1 and c % 2 == 0:  # the receive is posted at layer 77 (38's place in stage 0) ...
                assert fwd.recvs == [(0, 38, 77)]
                fwd.hook("mla_prep", 77, True)
            fwd.end_call()  # ... or, on odd calls, when the call ends
        fwd.drain()
        if rank == 1:  # the last call's picks
            a, t = fwd.received(38)
            got.append((int(a[0]), int(a[-1]), int(t[0])))
        fwd.close()
        gd.barrier()
        gd.finish()
        q.put((rank, "ok", got, fwd.bytes_per_call))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", f"{type(e).__name__}: {str(e)[:200]}", None))
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def test_two_ranks_forward_the_picks_every_call():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_forward_main, args=(r, 2, port, q, 3)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=120)
        assert not p.is_alive(), "a rank hung"
    res = sorted((q.get() for _ in range(2)), key=lambda x: x[0])
    assert [r[1] for r in res] == ["ok", "ok"], res
    T = 16
    assert res[1][2] == [(1000 * c, T * 2048 - 1 + 1000 * c, c + 1) for c in range(3)]
    assert res[0][3] == res[1][3] == stage.picks_bytes(T)
