"""The C oracle on its own (no GPU): conversions against ml_dtypes, known answers worked out by hand
from the reference's formulas, and -- the pin -- the reference kernels' own outputs recorded on a B200
(tests/golden, written by tests/golden/make_golden.py)."""
import hashlib
import json
import pathlib

import numpy as np
import pytest

from compare import assert_equal, assert_prep_close
from glmkv import workload as W
from layer_case import LayerCase, run_oracle
from oracle import cpu

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


# ------------------------------------------------------------------------------------------ formats

def test_e4m3_satfinite_matches_ml_dtypes():
    ml = pytest.importorskip("ml_dtypes")
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(1 << 18).astype(np.float32) * s for s in (1e-4, 1e-2, 1, 30, 300, 1e3)])
    x = np.concatenate([x, np.float32([0, -0.0, 448, 449, 463.9, 464, 465, -480, 1e30, np.inf, -np.inf,
                                       2 ** -10, 2 ** -10 * 1.0001, 3 * 2 ** -11, 2 ** -9, 2 ** -6])])
    want = np.clip(x, -448, 448).astype(ml.float8_e4m3fn).view(np.uint8)
    assert_equal(cpu.e4m3_from_f32(x), want, "e4m3 satfinite")


def test_e4m3_decode_and_bf16_round():
    ml = pytest.importorskip("ml_dtypes")
    codes = np.arange(256, dtype=np.uint8)
    got = cpu.f32_from_e4m3(codes)
    want = codes.view(ml.float8_e4m3fn).astype(np.float32)
    assert np.array_equal(got, want, equal_nan=True)
    x = np.random.default_rng(1).standard_normal(1 << 20).astype(np.float32) * 100
    assert_equal(cpu.bf16_from_f32(x), x.astype(ml.bfloat16).view(np.uint16), "bf16 RNE")
    assert_equal(cpu.bf16_from_f32(np.float32([np.nan, -np.nan])), np.uint16([0x7FFF, 0x7FFF]), "bf16 NaN")


# ------------------------------------------------------------------------------------------ known answers

def test_plan_known_answer():
    """Two sequences: lengths 5 and 70 with 2 and 3 fresh rows (glm_glue.cu:109-125)."""
    cu = np.int64([0, 2, 5])
    lens = np.int32([5, 70])
    T = 5
    out = {k: np.zeros(T, np.int32) for k in ("pos", "klen", "row_seq", "zero")}
    ks, ke = np.zeros(T, np.uint32), np.zeros(T, np.uint32)
    out["zero"][:] = 9
    cpu.plan(cu, lens, 2, out["pos"], ks, ke, out["klen"], out["row_seq"], out["zero"], T)
    assert out["pos"].tolist() == [3, 4, 67, 68, 69]
    assert ks.tolist() == [0, 0, 5, 5, 5]
    assert ke.tolist() == [4, 5, 73, 74, 75]
    assert out["klen"].tolist() == [4, 5, 68, 69, 70]
    assert out["row_seq"].tolist() == [0, 0, 1, 1, 1]
    assert out["zero"].tolist() == [0] * 5


def test_topk_known_answer():
    ind = np.full((2, 2048), -1, np.int32)
    ind[0, :3] = [0, 7, 2]
    ind[1, :4] = [64, 65, 0, 129]
    ind[1, 4] = -5
    s = ind.copy()
    cpu.topk_stream(s, np.uint32([100, 1000]), np.int32([3, 5000]), tl := np.zeros(2, np.int32), 2)
    assert s[0, :4].tolist() == [100, 107, 102, -1] and s[1, :5].tolist() == [1064, 1065, 1000, 1129, -1]
    assert tl.tolist() == [3, 2048]
    bt = np.int32([[9, 4, 7], [2, 5, 3]])
    s = ind.copy()
    cpu.topk_slots(s, bt, 3, np.int32([1, 0]), np.int32([3, 130]), tl, 2)
    assert s[0, :3].tolist() == [2 * 64, 2 * 64 + 7, 2 * 64 + 2]
    assert s[1, :5].tolist() == [4 * 64, 4 * 64 + 1, 9 * 64, 7 * 64 + 1, -1]
    assert tl.tolist() == [3, 130]


def test_dequant_known_answer():
    """One page, two rows: e4m3 0x38 (1.0), 0x40 (2.0), 0xB8 (-1.0), 0x01 (2^-9) times tile scales."""
    kv = np.zeros(64 * 656, np.uint8).reshape(64, 656)
    kv[0, 0], kv[0, 1], kv[0, 128], kv[0, 511] = 0x38, 0x40, 0xB8, 0x01
    kv[0, 512:528] = np.float32([3.0, 0.5, 1.0, 2.0 ** 20]).view(np.uint8)
    kv[0, 528:656] = np.arange(128, dtype=np.uint8)
    kv[1, 0] = 0x7F  # NaN code
    kv[1, 512:528] = np.float32([1, 1, 1, 1]).view(np.uint8)
    out = np.zeros(2 * 576, np.uint16)
    cpu.kv_dequant(kv.reshape(-1), np.int32([[0]]), 1, np.int32([2]), 1, out)
    o = out.reshape(2, 576)
    assert o[0, 0] == 0x4040 and o[0, 1] == 0x40C0      # 3.0, 6.0
    assert o[0, 128] == 0xBF00                           # -0.5
    assert o[0, 511] == 0x4500                           # 2^-9 * 2^20 = 2^11
    assert o[0, 2] == 0 and o[1, 0] == 0x7FFF
    assert_equal(o[0, 512:].view(np.uint8), np.arange(128, dtype=np.uint8), "k_pe verbatim")


def test_ue8m0_and_quant_known_answer():
    """A q_a row whose normalised values are exact: rows of +-1 with g_q = 1 give rms 1 / sqrt(1 + 1e-5)."""
    call = W.make_call([0], [1], np.random.default_rng(0))
    case = LayerCase(call, "fp8", seed=0, with_topk=False)
    case.x[:] = W.bf16_bits(np.ones((1, case.lda), np.float32))
    case.w.g_q[:] = W.bf16_bits(np.ones(2048, np.float32))
    h = case.host()
    run_oracle(case, h, full=False)
    # y = bf16(1 * rq) = bf16(0.999995) = 1.0 -> amax 1.0, scale 2^ceil(log2(1/448)) = 2^-8 (exponent byte 119)
    assert np.all(h["qsf"][:16] == 119)
    assert np.all(h["qq"][:2048] == cpu.e4m3_from_f32(np.float32([256.0]))[0])


def test_q_post_known_answer():
    """cos 1 / sin 0 leaves q_pe as it is; an indexer head whose largest value is 448 has scale 1."""
    T, ldb = 1, 64 * 256 + 32 * 128
    qb = np.zeros((T, ldb), np.uint16)
    qb[0, 192:256] = W.bf16_bits(np.arange(64, dtype=np.float32) - 32)          # head 0's q_pe
    qb[0, 16384:16384 + 128] = W.bf16_bits(np.linspace(-448, 448, 128, dtype=np.float32))
    rope = np.zeros((1, 64), np.uint16)
    rope[0, :32] = W.bf16_bits(np.ones(32, np.float32))
    qmla = np.zeros(64 * 576, np.uint16)
    iq = np.zeros(32 * 128, np.uint8)
    iw = W.bf16_bits(np.full(32, 2.0, np.float32))
    wout = np.zeros(32, np.float32)
    cpu.q_post(qb, ldb, rope, np.int32([0]), qmla, iq, iw, wout, 1, T)
    assert_equal(qmla[512:576], qb[0, 192:256], "q_pe through an identity rope")
    vals = np.linspace(-448, 448, 128, dtype=np.float32)
    assert_equal(iq[:128], cpu.e4m3_from_f32(W.bf16_value(W.bf16_bits(vals))), "head 0 at scale 1")
    assert wout[0] == np.float32(np.float32(np.float32(2.0 * 1.0) * np.float32(0.08838834764831845)) *
                                 np.float32(0.17677669529663687))
    assert np.all(wout[1:] == wout[1])  # all-zero heads: scale from eps 1e-4


# ------------------------------------------------------------------------------------------ pinned to the reference

def _small_case(name):
    import sys
    sys.path.insert(0, str(GOLDEN))
    import make_golden as MG

    spec = {s[0]: s for s in MG.SMALL}[name]
    _, cfg, cseed, seed, kv_dtype, full, zt = spec
    case = LayerCase(MG.call_of(cfg, cseed), kv_dtype=kv_dtype, seed=seed, zero_tiles=zt)
    return MG, case, full


@pytest.mark.parametrize("name", ["fp8_full", "fp8_shared", "bf16_full"])
def test_oracle_matches_reference_small(name):
    path = GOLDEN / f"ref_small_{name}.npz"
    if not path.exists():
        pytest.skip("golden vectors not generated yet (tests/golden/make_golden.py on a GPU)")
    ref = np.load(path)
    MG, case, full = _small_case(name)
    assert str(ref["input_sha"]) == MG.input_digest(case), "input generator drifted from the recorded vectors"
    h = case.host()
    run_oracle(case, h, full)
    for k in ("pos", "ks", "ke", "klen", "row_seq", "zero", "ind", "tlen"):
        if k in ref.files and h.get(k) is not None:
            assert_equal(h[k], ref[k].view(h[k].dtype), f"{name}: {k}")
    kv, keys, scs = MG.fresh_cache_rows(case, {"kv": h["kv"], "idx": h["idx"]})
    # append outputs within the rsqrtf tolerance; the reference's fresh rows then feed exact checks
    want = {"qq": ref["qq"], "qsf": ref["qsf"], "kv": h["kv"].copy(), "idx": h["idx"].copy()}
    row = 656 if case.kv_dtype == "fp8" else 1152
    want["kv"].reshape(-1, row)[case.call.slot_mapping] = ref["kv_fresh"]
    pages = want["idx"].reshape(-1, 64 * 132)
    for s, k_, sc in zip(case.call.slot_mapping, ref["idx_keys_fresh"], ref["idx_sc_fresh"]):
        pages[s // 64, (s % 64) * 128:(s % 64) * 128 + 128] = k_
        pages[s // 64, 8192 + 4 * (s % 64):8196 + 4 * (s % 64)] = sc
    assert_prep_close(h, want, case, full, what=f"{name} oracle vs reference")
    # the gather / dequant of the reference's cache state: bit-exact
    if full:
        kg, ksf = np.zeros_like(h["kg"]), np.zeros_like(h["ksf"])
        c = case.call
        cpu.idx_gather(want["idx"], c.block_table, c.max_pages, c.seq_lens, c.nseq, kg, ksf)
        assert_equal(kg, ref["kg"], f"{name}: kg")
        assert_equal(ksf.view(np.uint32), ref["ksf"].view(np.uint32), f"{name}: ksf")
    if case.kv_dtype == "fp8":
        kvd = np.zeros_like(h["kvd"])
        c = case.call
        cpu.kv_dequant(want["kv"], c.block_table, c.max_pages, c.seq_lens, c.nseq, kvd)
        assert_equal(kvd, ref["kvd"].view(np.uint16), f"{name}: kvd")


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("name", ["cfg0_fp8_full", "cfg4_fp8_full", "cfg4_bf16_full", "cfg1_fp8_full"])
def test_oracle_matches_reference_digests(name):
    path = GOLDEN / "ref_digests.json"
    if not path.exists():
        pytest.skip("golden vectors not generated yet (tests/golden/make_golden.py on a GPU)")
    want = json.loads(path.read_text())[name]
    import sys
    sys.path.insert(0, str(GOLDEN))
    import make_golden as MG

    spec = {s[0]: s for s in MG.DIGEST}[name]
    _, cfg, cseed, seed, kv_dtype, full, zt = spec
    case = LayerCase(MG.call_of(cfg, cseed), kv_dtype=kv_dtype, seed=seed, zero_tiles=zt)
    assert want["input_sha"] == MG.input_digest(case), "input generator drifted from the recorded vectors"
    h = case.host()
    run_oracle(case, h, full)
    for k in MG.EXACT:
        if k in want:
            assert _sha(h[k]) == want[k], f"{name}: {k}"
    pr = MG.prefix_rows(case.call)
    if "kvd_prefix" in want:
        assert _sha(h["kvd"].reshape(-1, 576)[pr]) == want["kvd_prefix"], f"{name}: kvd prefix rows"
    if "kg_prefix" in want:
        assert _sha(h["kg"].reshape(-1, 128)[pr]) == want["kg_prefix"], f"{name}: kg prefix rows"
        assert _sha(h["ksf"][pr]) == want["ksf_prefix"], f"{name}: ksf prefix rows"


@pytest.mark.parametrize("name", ["q_post_full", "q_post_shared"])
def test_oracle_q_post_matches_reference_digests(name):
    path = GOLDEN / "ref_digests.json"
    want = json.loads(path.read_text()) if path.exists() else {}
    if name not in want:
        pytest.skip("q_post golden vectors not generated yet (tests/golden/make_golden.py on a GPU)")
    want = want[name]
    import sys
    sys.path.insert(0, str(GOLDEN))
    import make_golden as MG
    from layer_case import q_post_case

    _, T, seed, full = {q[0]: q for q in MG.Q_POST}[name]
    c = q_post_case(T, seed)
    assert want["input_sha"] == MG.q_post_input_digest(c), "input generator drifted from the recorded vectors"
    qmla = np.zeros(T * 64 * 576, np.uint16)
    iq = np.zeros(T * 32 * 128, np.uint8)
    wout = np.zeros(T * 32, np.float32)
    cpu.q_post(c["qb"], c["ldb"], c["rope"], c["pos"], qmla, iq if full else None, c["iw"] if full else None,
               wout if full else None, full, T)
    assert _sha(qmla.reshape(T, 64, 576)[:, :, 512:]) == want["qmla_tails"]
    assert _sha(iq) == want["iq"]
    assert _sha(wout.view(np.uint32)) == want["wout"]


@pytest.mark.parametrize("name", ["quant_640", "quant_16384"])
def test_oracle_quant_matches_reference_digests(name):
    path = GOLDEN / "ref_digests.json"
    want = json.loads(path.read_text()) if path.exists() else {}
    if name not in want:
        pytest.skip("glm_quant golden vectors not generated yet (tests/golden/make_golden.py on a GPU)")
    import sys
    sys.path.insert(0, str(GOLDEN))
    import make_golden as MG
    from layer_case import quant_case

    _, T, K, ldx = {q[0]: q for q in MG.QUANT}[name]
    x = quant_case(T, K, ldx)
    assert want[name]["input_sha"] == _sha(x), "input generator drifted from the recorded vectors"
    q = np.zeros(T * K, np.uint8)
    sf = np.zeros((K + 511) // 512 * T * 4, np.uint8)
    cpu.quant(x, ldx, q, sf, T, K, T)
    assert _sha(q) == want[name]["q"] and _sha(sf) == want[name]["sf"]


@pytest.mark.parametrize("name", ["norm_add", "norm_noadd"])
def test_oracle_add_rms_quant_matches_reference(name):
    from compare import BF16_REL, E4M3_REL, assert_values_close, bf16_to_f32
    path = GOLDEN / f"ref_small_{name}.npz"
    if not path.exists():
        pytest.skip("glm_add_rms_quant golden vectors not generated yet (tests/golden/make_golden.py on a GPU)")
    ref = np.load(path)
    import sys
    sys.path.insert(0, str(GOLDEN))
    import make_golden as MG
    from layer_case import norm_case

    _, T, seed, with_a = {n[0]: n for n in MG.NORM_SMALL}[name]
    a, res, gamma = norm_case(T, seed, with_a)
    normed = np.zeros(T * 6144, np.uint16)
    q = np.zeros(T * 6144, np.uint8)
    sf = np.zeros(12 * T * 4, np.uint8)
    cpu.add_rms_quant(a, res, gamma, normed, q, sf, T, T)
    assert_equal(res.reshape(-1), ref["res"].reshape(-1), f"{name}: res")
    assert_values_close(bf16_to_f32(normed), bf16_to_f32(ref["normed"]), BF16_REL, f"{name}: normed")

    def vals(qq, ss):
        e = ss.reshape(12, T, 4).transpose(1, 0, 2).reshape(T, 48).astype(np.int32)
        return cpu.f32_from_e4m3(qq).reshape(T, 48, 128) * np.ldexp(1.0, e - 127)[:, :, None]
    assert_values_close(vals(q, sf), vals(ref["q"], ref["sf"]), E4M3_REL, f"{name}: q")


def test_mqa_oracle_against_a_direct_loop():
    """oracle/mqa.py (the restated fp8 MQA logits, read from the cache pages) against a plain loop over
    rows, heads and keys on a small paged call, and its e4m3 table against ml_dtypes."""
    import ml_dtypes

    from glmkv import workload as W
    from oracle import mqa

    codes = np.arange(256, dtype=np.uint8)
    ref = codes.view(ml_dtypes.float8_e4m3fn).astype(np.float64)
    same = (mqa.E4M3 == ref) | (np.isnan(mqa.E4M3) & np.isnan(ref))
    assert same.all()

    rng = np.random.default_rng(7)
    call = W.make_call([70, 0, 5], [3, 4, 2], rng, spare_pages=1)
    pool = np.empty((call.n_pages, 64 * 132), np.uint8)
    c = rng.integers(0, 256, size=(call.n_pages, 8192), dtype=np.uint8)
    pool[:, :8192] = np.where((c & 0x7F) == 0x7F, c - 1, c)
    pool[:, 8192:] = np.exp2(rng.integers(-6, 3, size=(call.n_pages, 64))).astype(np.float32).view(np.uint8)
    R = call.T
    iq = rng.integers(0, 126, size=R * 32 * 128, dtype=np.uint8)
    w = rng.standard_normal((R, 32)).astype(np.float32)
    row_seq = np.repeat(np.arange(call.nseq, dtype=np.int32), call.fresh)
    klen = (W.positions(call) + 1).astype(np.int32)
    got = mqa.mqa_logits_paged(iq, pool, call.block_table, call.max_pages, row_seq, klen, w)
    q = mqa.E4M3[iq.reshape(R, 32, 128)]
    for r in range(R):
        s = row_seq[r]
        for p in range(klen[r]):
            page, row = call.block_table[s, p // 64], p % 64
            k = mqa.E4M3[pool[page, row * 128:(row + 1) * 128]]
            sc = float(pool[page, 8192 + 4 * row:8196 + 4 * row].view(np.float32)[0])
            want = sum(float(w[r, h]) * max(float(q[r, h] @ k) * sc, 0.0) for h in range(32))
            lg, mg = got[r]
            assert abs(lg[p] - want) <= 1e-12 * max(mg[p], 1e-30), (r, p)
