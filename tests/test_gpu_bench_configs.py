"""GPU parity on the configurations the benchmark times, at their full sizes, against the reference's
own glue kernels (kern-glm53 source/glm_glue.cu:202-444, compiled unmodified for sm_100a), bit for
bit:

* the bench's cfg3 call (seed 0: 16 sequences, 16,384 fresh rows, 548,864 stream tokens) through the
  largest stage of the 8-GPU placement, layers 42..53 (indexer layers 42, 46, 50 and nine shared
  layers), with the bench's own seeded caches, activations and top-k picks. ``LayerGroup.run_call``
  runs it; the reference kernels run the same program in the manifest's order (scripts/gen.py:323-398).
  Every layer's latent cache, indexer cache, dequantized stream, q quant, key gather and row plan is
  compared, on the device;
* the 16,384-row append of cfg2 into a 2^20-token page pool (one sequence, prefix 1,032,192), fp8 and
  bf16 latent caches, on an indexer layer.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _same(a, b):
    """Bitwise equality of two device tensors of any dtype."""
    return a.shape == b.shape and torch.equal(a.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8))


def test_bench_cfg3_largest_stage_matches_reference(cuda, ref):
    import bench
    import glmkv
    from glmkv import stage, workload as W

    call = W.config("cfg3", seed=0)
    assert (call.T, call.nseq, call.ctx) == (16384, 16, 548864)
    rank, world = 5, 8
    first, last = stage.group_of(rank, world, T=call.T, ctx=call.ctx)
    assert (first, last) == (42, 54)
    groups = [stage.LayerGroup(first, last, n_pages=call.n_pages, max_ctx=call.ctx, chunk=call.T, device=cuda)
              for _ in range(2)]
    mine, theirs = groups
    rope = torch.from_numpy(W.rope_table(int(call.seq_lens.max())).view(np.int16)).to(cuda).view(torch.bfloat16)
    gen = torch.Generator(device=cuda).manual_seed(1000 * 0 + rank)  # the bench's generator of this rank
    bench.fill_caches(torch, mine, gen)
    inputs = bench.layer_inputs(torch, mine, call.T, gen)
    picks = bench.topk_picks(torch, call, mine, gen)
    for g in groups:
        g.rope = rope
    for l in mine.layers:
        theirs.kv[l].copy_(mine.kv[l])
        if l in stage.FULL:
            theirs.idx[l].copy_(mine.idx[l])
    ind = [{l: v.clone() for l, v in picks.items()} for _ in range(2)]
    meta = bench.device_call(torch, call, cuda)

    # the reference, kernel by kernel; each layer's outputs kept before the next layer overwrites them
    want = {}

    def keep(l, before):
        if before:  # the append (and on indexer layers the gather and row plan) is done
            want[l] = {"qq": theirs.qq.clone(), "qsf": theirs.qsf.clone()}
            if l in stage.FULL:
                want[l].update(kg=theirs.kg[:call.ctx * 128].clone(), ksf=theirs.ksf[:call.ctx].clone())
        else:
            want[l]["kvd"] = theirs.kvd[:call.ctx * 576].clone()

    bench.run_call_reference(theirs, meta, inputs, ind[1], call.ctx, on_dequant=keep)
    torch.cuda.synchronize()

    bad = []

    def check(l, before):
        torch.cuda.synchronize()
        w = want[l]
        names = (("qq", "qsf") + (("kg", "ksf") if l in stage.FULL else ())) if before else ("kvd",)
        for k in names:
            got = getattr(mine, k)
            got = got[:w[k].numel()]
            if not _same(got, w[k]):
                bad.append(f"layer {l}: {k}")

    glmkv.fault_flags(clear=True)
    mine.run_call(meta, inputs, ind[0], on_dequant=check)
    torch.cuda.synchronize()
    assert glmkv.fault_flags() == 0
    assert not bad, bad
    for l in mine.layers:
        assert _same(mine.kv[l], theirs.kv[l]), f"layer {l}: latent cache"
        if l in stage.FULL:
            assert _same(mine.idx[l], theirs.idx[l]), f"layer {l}: indexer cache"
            assert _same(ind[0][l], ind[1][l]), f"layer {l}: row plan"
    for k in ("pos", "ks", "ke", "klen", "row_seq", "zero", "tlen"):
        assert _same(getattr(mine, k), getattr(theirs, k)), k
    # the picks really were remapped: every non-negative entry is a stream row of its own sequence
    ks = mine.ks.to(torch.int64)
    for l in picks:
        got = ind[0][l].to(torch.int64)
        live = got >= 0
        assert torch.all(got[live] >= ks[:, None].expand_as(got)[live])


@pytest.mark.parametrize("kv_dtype", ["fp8", "bf16"])
def test_cfg2_append_16384_rows_on_a_1m_token_pool(cuda, ref, kv_dtype):
    import glmkv
    from glmkv import workload as W
    from layer_case import LayerCase

    call = W.config("cfg2", seed=17)
    assert call.ctx == 1 << 20 and call.T == 16384
    case = LayerCase(call, kv_dtype=kv_dtype, seed=17, zero_tiles=64, with_topk=False)
    d = [case.device(torch, cuda) for _ in range(2)]
    c, T = call, call.T
    p = lambda x, k: x[k].data_ptr()
    for i, x in enumerate(d):
        if i == 0:
            glmkv.plan(x["cu"], x["seq_lens"], c.nseq, x["pos"], x["ks"], x["ke"], x["klen"], x["row_seq"], x["zero"],
                       T)
            glmkv.mla_prep_full(x["x"], case.lda, x["g_q"], x["g_kv"], x["rope"], x["pos"], x["slot"], x["kv"],
                                x["idx"], x["ik_w"], x["ik_b"], x["qq"], x["qsf"], case.sf_rows, T, kv_dtype=kv_dtype)
        else:
            ref.plan(p(x, "cu"), p(x, "seq_lens"), c.nseq, p(x, "pos"), p(x, "ks"), p(x, "ke"), p(x, "klen"),
                     p(x, "row_seq"), p(x, "zero"), T)
            ref.mla_prep(kv_dtype == "fp8", p(x, "x"), case.lda, p(x, "g_q"), p(x, "g_kv"), p(x, "rope"), p(x, "pos"),
                         p(x, "slot"), p(x, "kv"), p(x, "idx"), p(x, "ik_w"), p(x, "ik_b"), p(x, "qq"), p(x, "qsf"),
                         case.sf_rows, T)
    torch.cuda.synchronize()
    assert glmkv.fault_flags() == 0
    for k in ("pos", "ks", "ke", "klen", "row_seq", "zero", "qq", "qsf", "kv", "idx"):
        assert _same(d[0][k], d[1][k]), f"cfg2 append {kv_dtype}: {k}"
    # the append wrote its 16,384 fresh slots (and nothing else) into the 2^20-token pool
    row = 656 if kv_dtype == "fp8" else 1152
    pool = torch.from_numpy(case.kv_pool).to(cuda).view(-1, row)
    slots = torch.from_numpy(call.slot_mapping).to(cuda)
    changed = torch.any(d[0]["kv"].view(-1, row) != pool, dim=1)
    assert not torch.any(changed[torch.ones(pool.shape[0], dtype=torch.bool, device=cuda).index_fill_(0, slots, False)])
