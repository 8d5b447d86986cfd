"""The row-selective lift: glm_mark_rows (the bitmap of the stream rows a call's picks name) and
glm_kv_dequant_marked (the lift of those rows only), against the reference's own full lift
(kern-glm53 source/glm_glue.cu:378-414, compiled unmodified): every marked row bit-exact, every
other row of the stream untouched, and the bitmap equal to the set of picks computed on the host.
glm_topk_stream_mark (the row plan and the mark in one pass) must give the reference's
glm_topk_stream output (glm_glue.cu:416-428) and glm_mark_rows' bitmap, bit for bit.
FlashMLA reads only the picked rows (kern-glm53 README.md:30-31, scripts/gen.py:399-400), so these
are the rows its attention sees."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

SENTINEL = 0x7E57  # a bf16 pattern the lift never writes into an untouched row


def _stream_picks(call, ind_rel):
    """Sequence-relative picks -> stream rows (glm_topk_stream's arithmetic), -1 kept."""
    goff = np.concatenate([[0], np.cumsum(call.seq_lens)[:-1]]).astype(np.int64)
    row_seq = np.repeat(np.arange(call.nseq), call.fresh)
    ks = goff[row_seq]
    return np.where(ind_rel >= 0, ind_rel + ks[:, None], -1).astype(np.int32)


def _host_mask(picks, words):
    m = np.zeros(words * 64, bool)
    v = picks[picks >= 0]
    m[v] = True
    return m


def _run(cuda, ref, call, seed, ind_rel, nan_codes=False):
    import glmkv
    from layer_case import LayerCase

    case = LayerCase(call, "fp8", seed=seed, with_topk=False, nan_codes=nan_codes)
    d = case.device(torch, cuda)
    c, T = call, call.T
    glmkv.plan(d["cu"], d["seq_lens"], c.nseq, d["pos"], d["ks"], d["ke"], d["klen"], d["row_seq"], d["zero"], T)
    ind = torch.from_numpy(np.ascontiguousarray(ind_rel)).to(cuda)
    glmkv.topk_stream(ind, d["ks"], d["klen"], d["tlen"], T)
    words = (c.ctx + 63) // 64
    mask = torch.empty(words, dtype=torch.int64, device=cuda).fill_(-1)  # the launcher clears it
    glmkv.fault_flags(clear=True)
    glmkv.mark_rows(ind, d["ks"], d["ke"], T, mask, words)
    out = torch.full((c.ctx * 576,), 0, dtype=torch.int16, device=cuda).fill_(SENTINEL)
    glmkv.kv_dequant_marked(d["kv"], d["block_table"], c.max_pages, d["seq_lens"], c.nseq, mask,
                            out.view(torch.bfloat16))
    full = torch.zeros(c.ctx * 576, dtype=torch.bfloat16, device=cuda)
    ref.kv_dequant(d["kv"].data_ptr(), d["block_table"].data_ptr(), c.max_pages, d["seq_lens"].data_ptr(), c.nseq,
                   full.data_ptr(), c.ctx)
    torch.cuda.synchronize()
    assert glmkv.fault_flags() == 0
    picks = ind.cpu().numpy()
    assert np.array_equal(picks, _stream_picks(call, ind_rel)), "the row plan"
    _check_fused(cuda, ref, d, T, ind_rel, ind, mask, words)
    want = _host_mask(picks, words)
    got_bits = np.unpackbits(mask.cpu().numpy().view(np.uint8), bitorder="little").astype(bool)
    assert np.array_equal(got_bits, want), "the mark bitmap"
    marked = want[:c.ctx]
    written = _written_rows(call, marked)
    o = out.view(-1, 576)
    f = full.view(torch.int16).view(-1, 576)
    wr = torch.from_numpy(written).to(cuda)
    assert torch.equal(o[wr], f[wr]), "lifted rows vs the reference's lift"
    assert torch.all(o[~wr] == SENTINEL), "rows that are not to be lifted were written"
    return float(marked.mean())


def _check_fused(cuda, ref, d, T, ind_rel, ind_stream, mask, words):
    """glm_topk_stream_mark on the same sequence-relative picks: the reference's row plan (ind, tlen)
    and glm_mark_rows' bitmap, bit for bit."""
    import glmkv

    want_ind = torch.from_numpy(np.ascontiguousarray(ind_rel)).to(cuda)
    want_tlen = torch.full((T,), -7, dtype=torch.int32, device=cuda)
    ref.topk_stream(want_ind.data_ptr(), d["ks"].data_ptr(), d["klen"].data_ptr(), want_tlen.data_ptr(), T)
    got_ind = torch.from_numpy(np.ascontiguousarray(ind_rel)).to(cuda)
    got_tlen = torch.full((T,), -7, dtype=torch.int32, device=cuda)
    got_mask = torch.empty(words, dtype=torch.int64, device=cuda).fill_(-1)  # the launcher clears it
    glmkv.topk_stream_mark(got_ind, d["ks"], d["klen"], got_tlen, T, d["ke"], got_mask, words)
    torch.cuda.synchronize()
    assert glmkv.fault_flags() == 0
    assert torch.equal(got_ind, want_ind), "fused row plan vs the reference's glm_topk_stream"
    assert torch.equal(got_ind, ind_stream), "fused row plan vs glm_topk_stream"
    assert torch.equal(got_tlen, want_tlen), "fused tlen vs the reference's"
    assert torch.equal(got_mask, mask), "fused bitmap vs glm_mark_rows"


def _written_rows(call, marked, dense=48, planned_seqs=1024):
    """The rows the marked lift writes: the marked ones, and every row of a page with `dense` or more
    marked rows (when the call has at most `planned_seqs` sequences)."""
    out = marked.copy()
    if call.nseq > planned_seqs:
        return out
    goff = np.concatenate([[0], np.cumsum(call.seq_lens)[:-1]])
    for s0, ln in zip(goff, call.seq_lens):
        for j in range(0, int(ln), 64):
            a, b = s0 + j, s0 + min(j + 64, int(ln))
            if marked[a:b].sum() >= dense:
                out[a:b] = True
    return out


def test_marked_lift_cfg0_uniform_picks(cuda, ref):
    from glmkv import workload as W

    call = W.config("cfg0", seed=31)
    ind = W.topk_indices(np.random.default_rng(31), call)
    frac = _run(cuda, ref, call, 31, ind, nan_codes=True)
    assert frac > 0.9  # uniform picks over short sequences name almost every row


def test_marked_lift_sliding_window_picks_skip_pages(cuda, ref):
    """Each row picks its 2048 latest positions (a sliding window): long prefixes are mostly unmarked,
    whole pages are skipped and partial pages copied from their first to their last marked row."""
    from glmkv import workload as W

    rng = np.random.default_rng(32)
    call = W.make_call([20000, 0, 5000, 70], [300, 129, 64, 1], rng, spare_pages=4)
    klen = W.positions(call).astype(np.int64) + 1
    ar = np.arange(2048)
    ind = np.where(ar[None, :] < klen[:, None], np.maximum(klen[:, None] - 2048, 0) + ar[None, :], -1)
    frac = _run(cuda, ref, call, 32, ind.astype(np.int32))
    assert 0.1 < frac < 0.5


def test_marked_lift_scattered_rows(cuda, ref):
    """Picks that mark single rows here and there: page spans that start and end mid-page, pages with
    one row, rows straddling the mask words (sequence starts not aligned to 64)."""
    from glmkv import workload as W

    rng = np.random.default_rng(33)
    call = W.make_call([1000, 37, 650], [40, 3, 21], rng, spare_pages=2)
    klen = W.positions(call).astype(np.int64) + 1
    ind = np.full((call.T, 2048), -1, np.int32)
    for r in range(call.T):
        k = int(klen[r])
        n = int(rng.integers(0, min(k, 9) + 1))
        ind[r, :n] = rng.choice(k, size=n, replace=False)
    _run(cuda, ref, call, 33, ind)


def test_marked_lift_cfg3_full_size(cuda, ref):
    """The bench's cfg3 call (548,864 stream rows) with uniform picks. A sequence with a 256K prefix and
    few fresh rows leaves many rows unpicked, so not every row is marked (about 87% at this seed)."""
    from glmkv import workload as W

    call = W.config("cfg3", seed=0)
    ind = W.topk_indices(np.random.default_rng(34), call)
    frac = _run(cuda, ref, call, 34, ind)
    assert 0.5 < frac < 1.0


def test_mark_flags_picks_past_the_bitmap(cuda):
    """A pick past mask_words * 64 is skipped and sets fault bit 4; the others are marked."""
    import glmkv

    T, words = 3, 4
    ind = torch.full((T, 2048), -1, dtype=torch.int32, device=cuda)
    ind[0, :3] = torch.tensor([0, 63, 64], dtype=torch.int32)
    ind[1, 0] = 255
    ind[2, 0] = 256  # past the 4 words
    ks = torch.zeros(T, dtype=torch.int32, device=cuda)
    ke = torch.full((T,), 256, dtype=torch.int32, device=cuda)
    mask = torch.zeros(words, dtype=torch.int64, device=cuda)
    glmkv.fault_flags(clear=True)
    glmkv.mark_rows(ind, ks, ke, T, mask, words)
    torch.cuda.synchronize()
    assert glmkv.fault_flags(clear=True) == 4
    m = mask.cpu().numpy().view(np.uint64)
    assert list(m) == [(1 << 0) | (1 << 63), 1, 0, 1 << 63]
    # the fused op on the same picks as sequence-relative ones (ks = 0): the same bitmap and flag
    tlen = torch.zeros(T, dtype=torch.int32, device=cuda)
    klen = torch.full((T,), 300, dtype=torch.int32, device=cuda)
    mask2 = torch.zeros(words, dtype=torch.int64, device=cuda)
    ind2 = ind.clone()
    glmkv.topk_stream_mark(ind2, ks, klen, tlen, T, ke, mask2, words)
    torch.cuda.synchronize()
    assert glmkv.fault_flags(clear=True) == 4
    assert torch.equal(mask2, mask) and torch.equal(ind2, ind)
    assert torch.all(tlen == 300)


def test_marked_lift_more_sequences_than_planned(cuda, ref):
    """More than 1,024 sequences: the lift walks the pages with the sequential cursor instead of its
    planned list; the result is the same."""
    from glmkv import workload as W

    rng = np.random.default_rng(35)
    n = 1100
    lens = rng.integers(1, 150, size=n)
    fresh = np.minimum(lens, rng.integers(1, 4, size=n))
    call = W.make_call(lens - fresh, fresh, rng, spare_pages=3)
    klen = W.positions(call).astype(np.int64) + 1
    ind = np.full((call.T, 2048), -1, np.int32)
    for r in range(call.T):
        k = int(klen[r])
        m = int(rng.integers(0, min(k, 5) + 1))
        ind[r, :m] = rng.choice(k, size=m, replace=False)
    _run(cuda, ref, call, 35, ind)
