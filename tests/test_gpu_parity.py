"""GPU parity: every op of libglmkv against the reference's own glue kernels (bit-exact) and the C
oracle (bit-exact; append outputs downstream of rsqrtf within the tolerance of tests/compare.py).

The reference kernels are kern-glm53 ``source/glm_glue.cu`` compiled from source for sm_100a
(``oracle/_ref/libglmref.so``, built by ``oracle/build.py``); they are launched with the manifest grids.
"""
import numpy as np
import pytest

from compare import assert_equal, assert_prep_close
from layer_case import LayerCase, run_glmkv, run_oracle, run_reference, to_host

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _run_both(case, cuda, full=True):
    """The layer through libglmkv and through the reference kernels, on separate device copies."""
    import glmkv

    d_mine, d_ref = case.device(torch, cuda), case.device(torch, cuda)
    run_glmkv(case, d_mine, full)
    run_reference(case, d_ref, full)
    torch.cuda.synchronize()
    assert glmkv.fault_flags() == 0
    return to_host(d_mine, torch), to_host(d_ref, torch)


def _assert_all_equal(got, want, what):
    for k in got:
        g, w = got[k], want[k]
        if k in ("ksf",):
            g, w = g.view(np.uint32), w.view(np.uint32)
        assert_equal(g, w, f"{what}: {k}")


CASES = [
    ("cfg0", "fp8", True, 0),
    ("cfg0", "fp8", False, 0),
    ("cfg4", "fp8", True, 4),
    ("cfg4", "bf16", True, 4),
    ("cfg4", "bf16", False, 4),
    ("cfg1", "fp8", True, 16),
    ("cfg1-bf16", "bf16", True, 16),
]


@pytest.mark.parametrize("name,kv_dtype,full,zero_tiles", CASES)
def test_layer_vs_reference_and_oracle(cuda, ref, name, kv_dtype, full, zero_tiles):
    from glmkv import workload as W

    call = W.config(name, seed=3)
    case = LayerCase(call, kv_dtype=kv_dtype, seed=11, zero_tiles=zero_tiles)
    got, want = _run_both(case, cuda, full)
    _assert_all_equal(got, want, f"{name}/{kv_dtype}/{'full' if full else 'shared'} vs reference")
    h = case.host()
    run_oracle(case, h, full)
    for k in ("pos", "ks", "ke", "klen", "row_seq", "zero") + (("ind", "tlen") if full else ()):
        assert_equal(got[k], h[k], f"{name} vs oracle: {k}")
    # the append: within the rsqrtf tolerance of the oracle
    assert_prep_close(got, h, case, full, what=f"{name} vs oracle")
    # gather and dequant of the device's own cache state (fresh rows included): bit-exact
    from oracle import cpu
    c = case.call
    if full:
        kg, ksf = np.zeros_like(h["kg"]), np.zeros_like(h["ksf"])
        cpu.idx_gather(got["idx"], c.block_table, c.max_pages, c.seq_lens, c.nseq, kg, ksf)
        assert_equal(got["kg"], kg, f"{name} vs oracle: kg")
        assert_equal(got["ksf"].view(np.uint32), ksf.view(np.uint32), f"{name} vs oracle: ksf")
    if kv_dtype == "fp8":
        kvd = np.zeros_like(h["kvd"])
        cpu.kv_dequant(got["kv"], c.block_table, c.max_pages, c.seq_lens, c.nseq, kvd)
        assert_equal(got["kvd"], kvd, f"{name} vs oracle: kvd")


@pytest.mark.parametrize("kv_dtype,full", [("fp8", True), ("fp8", False), ("bf16", True)])
def test_append_padding_rows_skip_the_caches(cuda, ref, kv_dtype, full):
    """Rows with slot < 0 (padding) still get their q quant but write no cache row (glm_glue.cu:231-232):
    bit-exact against the reference, and the caches equal the oracle's everywhere else."""
    from glmkv import workload as W
    from oracle import cpu

    call = W.config("cfg0", seed=3)
    call.slot_mapping[::7] = -1
    call.slot_mapping[-3:] = -1  # the last rows of the call, and so of the last warp's share
    case = LayerCase(call, kv_dtype=kv_dtype, seed=13)
    got, want = _run_both(case, cuda, full)
    _assert_all_equal(got, want, f"padding rows/{kv_dtype}/{'full' if full else 'shared'} vs reference")
    h = case.host()
    run_oracle(case, h, full)
    assert_prep_close(got, h, case, full, what="padding rows vs oracle")
    # every cache row but the live slots is the input pool, untouched
    row = 656 if kv_dtype == "fp8" else 1152
    live = call.slot_mapping[call.slot_mapping >= 0]
    untouched = np.setdiff1d(np.arange(call.n_pages * 64), live)
    assert_equal(got["kv"].reshape(-1, row)[untouched], case.kv_pool.reshape(-1, row)[untouched], "kv rows not written")
    if full:
        pages = got["idx"].reshape(-1, 64 * 132)
        keys = pages[:, :8192].reshape(-1, 128)
        assert_equal(keys[untouched], case.idx_pool.reshape(-1, 64 * 132)[:, :8192].reshape(-1, 128)[untouched],
                     "indexer keys not written")


def test_dequant_all_codes_vs_reference(cuda, ref):
    """Every e4m3 code (NaN included) and scales over 24 binades: identical bits to the reference."""
    from glmkv import workload as W
    import glmkv
    from oracle import cpu

    call = W.config("cfg1", seed=5)
    case = LayerCase(call, seed=5, nan_codes=True, with_topk=False)
    d1, d2 = case.device(torch, cuda), case.device(torch, cuda)
    c = call
    glmkv.kv_dequant(d1["kv"], d1["block_table"], c.max_pages, d1["seq_lens"], c.nseq, d1["kvd"])
    ref.kv_dequant(d2["kv"].data_ptr(), d2["block_table"].data_ptr(), c.max_pages, d2["seq_lens"].data_ptr(), c.nseq,
                   d2["kvd"].data_ptr(), c.ctx)
    torch.cuda.synchronize()
    a = d1["kvd"].view(torch.int16).cpu().numpy().view(np.uint16)
    b = d2["kvd"].view(torch.int16).cpu().numpy().view(np.uint16)
    assert_equal(a, b, "kvd vs reference")
    h = np.zeros(max(c.ctx, 1) * 576, np.uint16)
    cpu.kv_dequant(case.kv_pool, c.block_table, c.max_pages, c.seq_lens, c.nseq, h)
    assert_equal(a, h, "kvd vs oracle")


@pytest.mark.parametrize("op", ["kv_dequant", "idx_gather", "topk_stream", "plan"])
def test_full_size_1m_context_vs_reference(cuda, ref, op):
    """cfg2: one sequence of 2^20 tokens (16,384 pages, a 1.2 GB bf16 stream), bit-exact on the device."""
    from glmkv import workload as W
    import glmkv

    c = W.config("cfg2", seed=7)
    g = torch.Generator(device=cuda).manual_seed(7)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    bt, sl, cu = t(c.block_table), t(c.seq_lens), t(c.cu)
    if op == "kv_dequant":
        kv = torch.randint(0, 256, (c.n_pages * 64 * 656,), dtype=torch.uint8, device=cuda, generator=g)
        out = [torch.zeros(c.ctx * 576, dtype=torch.bfloat16, device=cuda) for _ in range(2)]
        glmkv.kv_dequant(kv, bt, c.max_pages, sl, c.nseq, out[0])
        ref.kv_dequant(kv.data_ptr(), bt.data_ptr(), c.max_pages, sl.data_ptr(), c.nseq, out[1].data_ptr(), c.ctx)
        torch.cuda.synchronize()
        assert torch.equal(out[0].view(torch.int16), out[1].view(torch.int16))
    elif op == "idx_gather":
        idx = torch.randint(0, 256, (c.n_pages * 8448,), dtype=torch.uint8, device=cuda, generator=g)
        kg = [torch.zeros(c.ctx * 128, dtype=torch.uint8, device=cuda) for _ in range(2)]
        ksf = [torch.zeros(c.ctx, dtype=torch.float32, device=cuda) for _ in range(2)]
        glmkv.idx_gather(idx, bt, c.max_pages, sl, c.nseq, kg[0], ksf[0])
        ref.idx_gather(idx.data_ptr(), bt.data_ptr(), c.max_pages, sl.data_ptr(), c.nseq, kg[1].data_ptr(),
                       ksf[1].data_ptr(), c.ctx)
        torch.cuda.synchronize()
        assert torch.equal(kg[0], kg[1]) and torch.equal(ksf[0].view(torch.int32), ksf[1].view(torch.int32))
    elif op == "topk_stream":
        T = c.T
        pos = torch.from_numpy(W.positions(c)).to(cuda)
        klen = pos + 1
        ks = torch.zeros(T, dtype=torch.int32, device=cuda)
        ind0 = (torch.rand(T, 2048, device=cuda, generator=g) * klen[:, None].float()).to(torch.int32)
        ind0[:, -7:] = -1
        ind = [ind0.clone(), ind0.clone()]
        tl = [torch.zeros(T, dtype=torch.int32, device=cuda) for _ in range(2)]
        glmkv.topk_stream(ind[0], ks, klen, tl[0], T)
        ref.topk_stream(ind[1].data_ptr(), ks.data_ptr(), klen.data_ptr(), tl[1].data_ptr(), T)
        torch.cuda.synchronize()
        assert torch.equal(ind[0], ind[1]) and torch.equal(tl[0], tl[1])
    else:
        T = c.T
        outs = [[torch.zeros(T, dtype=torch.int32, device=cuda) for _ in range(6)] for _ in range(2)]
        glmkv.plan(cu, sl, c.nseq, *outs[0][:3], *outs[0][3:], T)
        ref.plan(cu.data_ptr(), sl.data_ptr(), c.nseq, *[o.data_ptr() for o in outs[1]], T)
        torch.cuda.synchronize()
        for a, b in zip(*outs):
            assert torch.equal(a, b)
    import glmkv as _g
    assert _g.fault_flags() == 0


@pytest.mark.parametrize("kv_dtype", ["fp8", "bf16"])
def test_full_size_append_16384_rows_vs_reference(cuda, ref, kv_dtype):
    """cfg1's 16,384-row append on an indexer layer, bit-exact against the reference kernel."""
    from glmkv import workload as W

    call = W.config("cfg1", seed=9)
    case = LayerCase(call, kv_dtype=kv_dtype, seed=9, zero_tiles=32, with_topk=False)
    got, want = _run_both(case, cuda, full=True)
    _assert_all_equal(got, want, f"cfg1 append {kv_dtype}")


def test_append_then_dequant_round_trip(cuda):
    """Property: the dequantized stream at the fresh rows is the e4m3 rounding of kv_norm, k_pe intact."""
    from glmkv import workload as W
    from compare import bf16_to_f32

    call = W.config("cfg0", seed=13)
    case = LayerCase(call, "fp8", seed=13, with_topk=False)
    bf = LayerCase(call, "bf16", seed=13, with_topk=False)
    d8, d16 = case.device(torch, cuda), bf.device(torch, cuda)
    run_glmkv(case, d8, full=False)
    run_glmkv(bf, d16, full=False)
    torch.cuda.synchronize()
    kvd = d8["kvd"].view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1, 576)
    rows16 = d16["kv"].cpu().numpy().reshape(-1, 1152).view(np.uint16)
    # stream rows of the fresh tokens
    goff = np.concatenate([[0], np.cumsum(call.seq_lens)[:-1]])
    srows = np.concatenate([g + np.arange(p, p + f) for g, p, f in zip(goff, call.prefix, call.fresh)])
    ref_rows = rows16[call.slot_mapping]
    a = bf16_to_f32(kvd[srows, :512]).astype(np.float64)
    b = bf16_to_f32(ref_rows[:, :512]).astype(np.float64)
    tile_max = np.abs(b.reshape(-1, 4, 128)).max(axis=2, keepdims=True)
    tol = (np.maximum(np.abs(b).reshape(-1, 4, 128) * 2 ** -4, tile_max / 448 * 2 ** -9) + 1e-30).reshape(-1, 512)
    assert np.all(np.abs(a - b) <= tol * 1.01)
    assert_equal(kvd[srows, 512:], ref_rows[:, 512:], "k_pe through the round trip")


def test_dequant_idempotent_and_stream_order(cuda):
    """Two dequant launches give identical streams; stream rows follow sequence order."""
    from glmkv import workload as W
    import glmkv

    call = W.config("cfg4", seed=2)
    case = LayerCase(call, "fp8", seed=2, with_topk=False, nan_codes=False)
    d = case.device(torch, cuda)
    c = call
    glmkv.kv_dequant(d["kv"], d["block_table"], c.max_pages, d["seq_lens"], c.nseq, d["kvd"])
    first = d["kvd"].clone()
    glmkv.kv_dequant(d["kv"], d["block_table"], c.max_pages, d["seq_lens"], c.nseq, d["kvd"])
    torch.cuda.synchronize()
    assert torch.equal(first.view(torch.int16), d["kvd"].view(torch.int16))


def test_bad_page_is_skipped_and_flagged(cuda):
    """A negative page number inside a sequence is not read: that page's rows are left untouched,
    every other page is lifted, and the call raises fault bit 2."""
    from glmkv import workload as W
    import glmkv

    call = W.config("cfg0", seed=4)
    case = LayerCase(call, "fp8", seed=4, with_topk=False, nan_codes=False)
    d = case.device(torch, cuda)
    c = call
    glmkv.fault_flags(clear=True)
    bt = d["block_table"].clone()
    bt[1, 3] = -1  # page 3 of sequence 1: stream rows 1536 + 192 .. + 255
    sentinel = torch.full_like(d["kvd"], 7.0)
    glmkv.kv_dequant(d["kv"], bt, c.max_pages, d["seq_lens"], c.nseq, sentinel)
    good = torch.zeros_like(d["kvd"])
    glmkv.kv_dequant(d["kv"], d["block_table"], c.max_pages, d["seq_lens"], c.nseq, good)
    torch.cuda.synchronize()
    assert glmkv.fault_flags(clear=True) == 2
    s = sentinel.view(-1, 576)
    g = good.view(-1, 576)
    lo, hi = 1536 + 192, 1536 + 256
    assert torch.all(s[lo:hi] == 7.0)
    assert torch.equal(s[:lo].view(torch.int16), g[:lo].view(torch.int16))
    assert torch.equal(s[hi:c.ctx].view(torch.int16), g[hi:c.ctx].view(torch.int16))


@pytest.mark.parametrize("lda", [2756, 2760])
def test_append_rows_not_aligned_for_bulk_copy(cuda, ref, lda):
    """Rows whose start is not 16-byte aligned (lda % 8 != 0) take the direct-load path; lda 2760 the
    bulk-copy one. Both bit-exact against the reference."""
    from glmkv import workload as W

    call = W.config("cfg0", seed=8)
    case = LayerCase(call, "fp8", seed=8, zero_tiles=3, with_topk=False)
    wide = np.zeros((case.T, lda), np.uint16)
    wide[:, :case.x.shape[1]] = case.x
    wide[:, case.x.shape[1]:] = 0x7FC0  # padding columns: NaN if anything read them
    case.x, case.lda = wide, lda
    got, want = _run_both(case, cuda, full=True)
    _assert_all_equal(got, want, f"lda {lda}")
