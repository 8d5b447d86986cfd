"""GPU tests of the host-facing paths: the bounded-wait timeout, many-sequence calls, and a multi-layer
LayerGroup call against the reference kernels run layer by layer."""
import numpy as np
import pytest

from compare import assert_equal
from layer_case import to_host

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def test_bounded_wait_times_out_and_flags(cuda):
    """A wait on a barrier nothing completes ends after its limit with fault bit 1; the context stays usable."""
    import glmkv
    from glmkv import _lib

    glmkv.fault_flags(clear=True)
    waited = torch.zeros(1, dtype=torch.int32, device=cuda)
    _lib.call("glmkv_selftest_wait", 20_000_000, waited.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert glmkv.fault_flags(clear=True) == 1
    ns = int(waited.item()) & 0xffffffff
    assert 20_000_000 <= ns < 2_000_000_000
    x = torch.arange(10, device=cuda)  # the context still works
    assert int(x.sum()) == 45


def _many_seq_call(n, seed):
    from glmkv import workload as W
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, 200, size=n)
    fresh = np.minimum(lens, rng.integers(1, 8, size=n))
    return W.make_call(lens - fresh, fresh, rng, spare_pages=5)


@pytest.mark.parametrize("nseq", [257, 300])
def test_more_sequences_than_staged(cuda, ref, nseq):
    """More than 256 sequences: glm_plan continues its scan in global memory; the page cursors walk
    hundreds of sequences. Bit-exact against the reference."""
    from layer_case import LayerCase, run_glmkv, run_reference

    case = LayerCase(_many_seq_call(nseq, nseq), "fp8", seed=nseq, with_topk=True)
    a, b = case.device(torch, cuda), case.device(torch, cuda)
    run_glmkv(case, a, full=True)
    run_reference(case, b, full=True)
    torch.cuda.synchronize()
    ga, gb = to_host(a, torch), to_host(b, torch)
    for k in ga:
        assert_equal(ga[k].view(np.uint8), gb[k].view(np.uint8), f"{nseq} sequences: {k}")


def test_layer_group_matches_reference_layer_by_layer(cuda, ref):
    """LayerGroup.run_call over layers 0..6 (indexer layers 0, 1, 2, 6 and shared 3, 4, 5) gives the
    caches, streams and row plans of the reference kernels run in the manifest's order."""
    import glmkv
    from glmkv import stage, workload as W

    call = W.config("cfg0", seed=21)
    rng = np.random.default_rng(21)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    meta = stage.CallMeta(t(call.cu), t(call.seq_lens), t(call.block_table), t(call.slot_mapping), call.nseq, call.T,
                          call.ctx)
    groups = [stage.LayerGroup(0, 7, n_pages=call.n_pages, max_ctx=call.ctx, chunk=call.T, device=cuda)
              for _ in range(2)]
    rope = t(W.rope_table(int(call.seq_lens.max())).view(np.int16)).view(torch.bfloat16)
    inputs, ind = {}, {}
    for l in range(7):
        w = W.weights(rng)
        bf = lambda a: t(a.view(np.int16)).view(torch.bfloat16)
        inputs[l] = stage.LayerInputs(bf(W.activations(rng, call.T)), bf(w.g_q), bf(w.g_kv),
                                      bf(w.ik_w) if l in stage.FULL else None, bf(w.ik_b) if l in stage.FULL else None)
        if l in stage.FULL:
            ind[l] = t(W.topk_indices(rng, call))
    pool = W.random_latent_pages(rng, call.n_pages, "fp8")
    ipool = W.random_index_pages(rng, call.n_pages)
    inds = [{l: v.clone() for l, v in ind.items()} for _ in range(2)]
    for g in groups:
        g.rope = rope
        for l in g.kv:
            g.kv[l].copy_(t(pool))
        for l in g.idx:
            g.idx[l].copy_(t(ipool))
    mine, theirs = groups
    # glmkv: the whole group in one call; keep each layer's stream as the next layer overwrites it
    kvd_mine = {}
    mine.run_call(meta, inputs, inds[0], on_dequant=lambda l, before: None if before else
                  kvd_mine.__setitem__(l, mine.kvd.clone()))
    # reference: the same program, kernel by kernel
    p = lambda x: x.data_ptr()
    ref.plan(p(meta.cu), p(meta.seq_lens), call.nseq, p(theirs.pos), p(theirs.ks), p(theirs.ke), p(theirs.klen),
             p(theirs.row_seq), p(theirs.zero), call.T)
    kvd_ref = {}
    for l in range(7):
        a = inputs[l]
        full = l in stage.FULL
        ref.mla_prep(True, p(a.x), a.x.shape[1], p(a.g_q), p(a.g_kv), p(rope), p(theirs.pos), p(meta.slot),
                     p(theirs.kv[l]), p(theirs.idx[l]) if full else None, p(a.ik_w) if full else None,
                     p(a.ik_b) if full else None, p(theirs.qq), p(theirs.qsf), theirs.sf_rows, call.T)
        if full:
            ref.idx_gather(p(theirs.idx[l]), p(meta.block_table), call.max_pages, p(meta.seq_lens), call.nseq,
                           p(theirs.kg), p(theirs.ksf), call.ctx)
            ref.topk_stream(p(inds[1][l]), p(theirs.ks), p(theirs.klen), p(theirs.tlen), call.T)
        ref.kv_dequant(p(theirs.kv[l]), p(meta.block_table), call.max_pages, p(meta.seq_lens), call.nseq,
                       p(theirs.kvd), call.ctx)
        kvd_ref[l] = theirs.kvd.clone()
    torch.cuda.synchronize()
    for l in range(7):
        assert torch.equal(mine.kv[l], theirs.kv[l]), f"layer {l} latent cache"
        assert torch.equal(kvd_mine[l].view(torch.int16), kvd_ref[l].view(torch.int16)), f"layer {l} stream"
        if l in stage.FULL:
            assert torch.equal(mine.idx[l], theirs.idx[l]), f"layer {l} indexer cache"
            assert torch.equal(inds[0][l], inds[1][l]), f"layer {l} row plan"
    for k in ("pos", "ks", "ke", "klen", "row_seq", "zero", "tlen", "qq", "qsf", "kg", "ksf"):
        assert torch.equal(getattr(mine, k), getattr(theirs, k)), k
    assert glmkv.fault_flags() == 0
