"""glm_mqa_logits_paged, the indexer's fp8 MQA logits read straight from the indexer cache pages,
against the NumPy restatement of DeepGEMM's published fp8_mqa_logits (oracle/mqa.py).

DeepGEMM is absent from kern-glm53 (an empty submodule), so the oracle is the formula its tests use;
the dot products there are exact (float64), and the device's f32 tensor-core result must lie within
2^-14 of `magnitude` (the same sum over |.|) of it. Positions at or past a row's klen are not written.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = 2.0 ** -14


def _codes(rng, n):
    """e4m3 codes without the NaN codes (0x7F, 0xFF): what the append's satfinite conversion writes."""
    c = rng.integers(0, 256, size=n, dtype=np.uint8)
    return np.where((c & 0x7F) == 0x7F, c - 1, c).astype(np.uint8)


def _case(prefix, fresh, seed):
    from glmkv import workload as W

    rng = np.random.default_rng(seed)
    call = W.make_call(prefix, fresh, rng, spare_pages=2)
    pool = np.empty((call.n_pages, 64 * 132), np.uint8)
    pool[:, :8192] = _codes(rng, call.n_pages * 8192).reshape(call.n_pages, 8192)
    pool[:, 8192:] = np.exp2(rng.integers(-12, 4, size=(call.n_pages, 64))).astype(np.float32).view(np.uint8)
    R = call.T
    iq = _codes(rng, R * 32 * 128)
    w = rng.standard_normal((R, 32)).astype(np.float32)
    row_seq = np.repeat(np.arange(call.nseq, dtype=np.int32), call.fresh)
    klen = W.positions(call) + 1
    return call, pool.reshape(-1), iq, w, row_seq, klen.astype(np.int32)


def _run(cuda, call, pool, iq, w, row_seq, klen, stride):
    import glmkv

    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    R = len(row_seq)
    logits = torch.full((R * stride,), float("nan"), dtype=torch.float32, device=cuda)
    glmkv.mqa_logits_paged(t(iq), t(pool), call.n_pages, t(call.block_table), call.max_pages, t(row_seq), t(klen),
                           t(w), logits, stride, R)
    torch.cuda.synchronize()
    assert glmkv.fault_flags() == 0
    return logits.cpu().numpy().reshape(R, stride)


def _check(got, call, pool, iq, w, row_seq, klen, what):
    from oracle import mqa

    want = mqa.mqa_logits_paged(iq, pool, call.block_table, call.max_pages, row_seq, klen, w)
    worst = 0.0
    for r, (lg, mg) in enumerate(want):
        k = int(klen[r])
        g = got[r, :k].astype(np.float64)
        assert np.all(np.isfinite(g)), f"{what}: row {r} has non-finite logits"
        err = np.abs(g - lg) / np.maximum(mg, 1e-30)
        worst = max(worst, float(err.max()))
        assert err.max() <= TOL, f"{what}: row {r} position {int(err.argmax())}: {g[err.argmax()]} vs {lg[err.argmax()]}"
        assert np.all(np.isnan(got[r, k:])), f"{what}: row {r} wrote past klen"
    print(f"{what}: worst error {worst:.3g} of magnitude")


def test_mqa_logits_small_ragged(cuda):
    """Four sequences whose rows straddle the 8-row blocks; key counts across the 64-key page and
    128-key tile edges (1 .. 1509)."""
    case = _case([100, 0, 700, 1500, 63], [20, 37, 13, 9, 1], seed=81)
    call, pool, iq, w, row_seq, klen = case
    stride = int(klen.max()) + 5
    got = _run(cuda, *case, stride)
    _check(got, *case, "small")


def test_mqa_logits_cfg0(cuda):
    """cfg0 (two sequences, 1,024 rows, up to 3,584 keys a row)."""
    from glmkv import workload as W

    c0 = W.config("cfg0", seed=4)
    case = _case(c0.prefix, c0.fresh, seed=82)
    got = _run(cuda, *case, 4096)
    _check(got, *case, "cfg0")


def test_mqa_logits_stride_below_klen_and_sub_chunks(cuda):
    """A stride below some rows' klen keeps every store inside the row (positions >= stride are not
    written), and the rows scored in sub-chunks (the manifest's --sub) match one launch."""
    import glmkv

    case = _case([300, 0, 900], [40, 25, 19], seed=83)
    call, pool, iq, w, row_seq, klen = case
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    R, stride = len(row_seq), 640  # rows of the third sequence reach klen 919
    got = _run(cuda, *case, stride)
    from oracle import mqa
    want = mqa.mqa_logits_paged(iq, pool, call.block_table, call.max_pages, row_seq, klen, w)
    for r, (lg, mg) in enumerate(want):
        k = min(int(klen[r]), stride)
        err = np.abs(got[r, :k].astype(np.float64) - lg[:k]) / np.maximum(mg[:k], 1e-30)
        assert err.max() <= TOL, r
        assert np.all(np.isnan(got[r, k:])), r
    # the same rows in sub-chunks of 24 rows (block edges inside sequences), row pointers offset
    sub = torch.full((R * stride,), float("nan"), dtype=torch.float32, device=cuda)
    iq_d, w_d, rs_d, kl_d, bt_d, pool_d = t(iq), t(w), t(row_seq), t(klen), t(call.block_table), t(pool)
    for j in range(0, R, 24):
        n = min(24, R - j)
        glmkv.mqa_logits_paged(iq_d[j * 4096:], pool_d, call.n_pages, bt_d, call.max_pages, rs_d[j:], kl_d[j:],
                               w_d[j:], sub[j * stride:], stride, n)
    torch.cuda.synchronize()
    assert np.array_equal(sub.cpu().numpy().reshape(R, stride), got, equal_nan=True)


def test_mqa_logits_bad_page_is_flagged(cuda):
    """A block-table entry outside the pool is skipped (never read) and flagged; other sequences'
    logits are unaffected."""
    import glmkv

    case = _case([200, 130], [30, 20], seed=84)
    call, pool, iq, w, row_seq, klen = case
    bt = call.block_table.copy()
    bt[1, 1] = call.n_pages + 5  # sequence 1, positions 64 .. 127
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    R, stride = len(row_seq), 256
    logits = torch.full((R * stride,), float("nan"), dtype=torch.float32, device=cuda)
    glmkv.fault_flags()
    glmkv.mqa_logits_paged(t(iq), t(pool), call.n_pages, t(bt), call.max_pages, t(row_seq), t(klen), t(w), logits,
                           stride, R)
    torch.cuda.synchronize()
    assert glmkv.fault_flags() & 2
    got = logits.cpu().numpy().reshape(R, stride)
    from oracle import mqa
    want = mqa.mqa_logits_paged(iq, pool, call.block_table, call.max_pages, row_seq, klen, w)
    for r in range(R):
        if row_seq[r] == 0:  # sequence 0 reads only its own pages
            lg, mg = want[r]
            err = np.abs(got[r, :klen[r]] - lg) / np.maximum(mg, 1e-30)
            assert err.max() <= TOL, r


def test_mqa_logits_rejects_bad_arguments():
    import glmkv
    from glmkv import _lib

    L = glmkv.lib()
    A = 0x10000
    assert L.glmkv_mqa_logits_paged(A, A, 1, A, 1, A, A, A, A, 16, -1, None) == _lib.ERR_ARG
    assert L.glmkv_mqa_logits_paged(A, A, 0, A, 1, A, A, A, A, 16, 8, None) == _lib.ERR_ARG
    assert L.glmkv_mqa_logits_paged(A + 8, A, 1, A, 1, A, A, A, A, 16, 8, None) == _lib.ERR_ALIGN
    assert L.glmkv_mqa_logits_paged(A, A, 1, A, 1, A, A, A, A, 16, 0, None) == _lib.OK


def test_mqa_logits_full_size_cfg3(cuda):
    """The bench's cfg3 call at full size (16,384 rows, up to 262,912 keys a row), in the manifest's
    1,024-row sub-chunks: 16 rows spread over the call against the oracle, and the first 4,096 rows
    bit-identical to one 4,096-row launch (the logits do not depend on how the rows are split)."""
    import glmkv
    from glmkv import workload as W
    from oracle import mqa

    c3 = W.config("cfg3", seed=0)
    case = _case(c3.prefix, c3.fresh, seed=85)
    call, pool, iq, w, row_seq, klen = case
    R, stride, sub = len(row_seq), int(klen.max()), 1024
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    iq_d, w_d, rs_d, kl_d, bt_d, pool_d = t(iq), t(w), t(row_seq), t(klen), t(call.block_table), t(pool)

    def launch(out, j, n):
        glmkv.mqa_logits_paged(iq_d[j * 4096:], pool_d, call.n_pages, bt_d, call.max_pages, rs_d[j:], kl_d[j:],
                               w_d[j:], out, stride, n)

    sample = np.linspace(0, R - 1, 16).astype(int)
    got = {}
    first = torch.full((4096 * stride,), float("nan"), dtype=torch.float32, device=cuda)
    buf = torch.empty((sub * stride,), dtype=torch.float32, device=cuda)
    for j in range(0, R, sub):
        buf.fill_(float("nan"))
        launch(buf, j, sub)
        torch.cuda.synchronize()
        assert glmkv.fault_flags() == 0
        if j < 4096:
            first[j * stride:(j + sub) * stride].copy_(buf)
        for r in sample[(sample >= j) & (sample < j + sub)]:
            got[int(r)] = buf[(r - j) * stride:(r - j) * stride + int(klen[r])].cpu().numpy().astype(np.float64)
    whole = torch.full((4096 * stride,), float("nan"), dtype=torch.float32, device=cuda)
    launch(whole, 0, 4096)
    torch.cuda.synchronize()
    assert torch.equal(whole.view(torch.int32), first.view(torch.int32))
    del whole, first, buf

    rows = np.array(sorted(got))
    iq_rows = iq.reshape(R, 32 * 128)[rows]
    want = mqa.mqa_logits_paged(iq_rows, pool, call.block_table, call.max_pages, row_seq[rows], klen[rows], w[rows])
    worst = 0.0
    for r, (lg, mg) in zip(rows, want):
        err = np.abs(got[r] - lg) / np.maximum(mg, 1e-30)
        worst = max(worst, float(err.max()))
        assert err.max() <= TOL, f"row {r} position {int(err.argmax())}"
    print(f"cfg3: {len(rows)} rows up to {int(klen[rows].max())} keys, worst error {worst:.3g} of magnitude")


def test_mqa_logits_rows_without_keys(cuda):
    """Rows whose klen is 0 (no key yet) get no logits and leave the other rows of their block
    untouched; a launch where no row has a key writes nothing and flags nothing."""
    import glmkv

    case = _case([150, 0, 300], [12, 9, 7], seed=86)
    call, pool, iq, w, row_seq, klen = case
    klen = klen.copy()
    klen[[0, 5, 12, 13, 27]] = 0  # inside a block, a block's first row, a sequence's first rows, the last row
    R, stride = len(row_seq), 320
    got = _run(cuda, call, pool, iq, w, row_seq, klen, stride)
    from oracle import mqa
    want = mqa.mqa_logits_paged(iq, pool, call.block_table, call.max_pages, row_seq, klen, w)
    for r, (lg, mg) in enumerate(want):
        k = int(klen[r])
        assert np.all(np.isnan(got[r, k:])), r
        if k:
            err = np.abs(got[r, :k].astype(np.float64) - lg) / np.maximum(mg, 1e-30)
            assert err.max() <= TOL, r
    none = _run(cuda, call, pool, iq, w, row_seq, np.zeros_like(klen), stride)
    assert np.all(np.isnan(none))


def test_mqa_logits_partial_block_and_empty_segment(cuda):
    """R not a multiple of 8 (the last block's query tile is zero-filled past R), and blocks whose rows
    span two sequences where one whole segment has klen 0. Nothing is written for rows past R (a NaN
    guard region after the last row stays NaN) or for the empty segment's rows."""
    import glmkv

    case = _case([40, 0, 200], [5, 6, 10], seed=87)
    call, pool, iq, w, row_seq, klen = case
    klen = klen.copy()
    klen[row_seq == 1] = 0  # rows 5 .. 10: the second segment of block 0 and the first of block 1
    R, stride = len(row_seq), 224
    assert R % 8 != 0
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    logits = torch.full(((R + 8) * stride,), float("nan"), dtype=torch.float32, device=cuda)
    glmkv.mqa_logits_paged(t(iq), t(pool), call.n_pages, t(call.block_table), call.max_pages, t(row_seq), t(klen),
                           t(w), logits, stride, R)
    torch.cuda.synchronize()
    assert glmkv.fault_flags() == 0
    got = logits.cpu().numpy().reshape(R + 8, stride)
    assert np.all(np.isnan(got[R:])), "logits written past the last row"
    from oracle import mqa
    want = mqa.mqa_logits_paged(iq, pool, call.block_table, call.max_pages, row_seq, klen, w)
    for r, (lg, mg) in enumerate(want):
        k = int(klen[r])
        assert np.all(np.isnan(got[r, k:])), r
        if k:
            err = np.abs(got[r, :k].astype(np.float64) - lg) / np.maximum(mg, 1e-30)
            assert err.max() <= TOL, r


def test_mqa_logits_keys_past_the_block_table_are_flagged(cuda):
    """Rows whose klen reaches past the block table's max_pages pages: those key pages are not read
    (no entry exists for them) and the launch sets fault bit 2; positions inside the table stay exact."""
    import glmkv

    case = _case([300], [20], seed=88)
    call, pool, iq, w, row_seq, klen = case
    mp = 3  # pages 0 .. 2 (positions < 192) of a sequence that reaches position 319
    bt = np.ascontiguousarray(call.block_table[:, :mp])
    R, stride = len(row_seq), 320
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    logits = torch.full((R * stride,), float("nan"), dtype=torch.float32, device=cuda)
    glmkv.fault_flags(clear=True)
    glmkv.mqa_logits_paged(t(iq), t(pool), call.n_pages, t(bt), mp, t(row_seq), t(klen), t(w), logits, stride, R)
    torch.cuda.synchronize()
    assert glmkv.fault_flags(clear=True) & 2
    got = logits.cpu().numpy().reshape(R, stride)
    from oracle import mqa
    want = mqa.mqa_logits_paged(iq, pool, call.block_table, call.max_pages, row_seq, klen, w)
    for r, (lg, mg) in enumerate(want):
        k = min(int(klen[r]), mp * 64)
        err = np.abs(got[r, :k].astype(np.float64) - lg[:k]) / np.maximum(mg[:k], 1e-30)
        assert err.max() <= TOL, r
