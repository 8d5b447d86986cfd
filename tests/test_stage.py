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
