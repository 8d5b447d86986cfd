"""Comparisons used by the parity tests.

Bit-exact everywhere except where the C oracle cannot be: it replaces CUDA's approximate rsqrtf with
the correctly rounded 1/sqrt, so the q_a / kv_a RMS factors and the indexer LayerNorm factor of a
row may land one or two f32 ulps apart. Outputs downstream of those factors are compared with
`assert_quant_close` against the oracle (and bit-exactly against the reference kernels).
"""
import numpy as np

E4M3_REL = 0.125          # one e4m3 code step relative to the value (3 mantissa bits)
BF16_REL = 2.0 ** -7      # one bf16 ulp relative
MAX_DIFF_FRAC = 2e-3      # at most this fraction of the elements may differ at all


def e4m3_to_f32(codes):
    from oracle import cpu
    return cpu.f32_from_e4m3(np.ascontiguousarray(codes, dtype=np.uint8))


def bf16_to_f32(bits):
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def assert_equal(got, want, what):
    got, want = np.asarray(got), np.asarray(want)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    if not np.array_equal(got, want):
        bad = np.flatnonzero(got.reshape(-1) != want.reshape(-1))
        i = bad[0]
        raise AssertionError(f"{what}: {len(bad)} of {got.size} elements differ; first at {i}: "
                             f"{got.reshape(-1)[i]} != {want.reshape(-1)[i]}")


def assert_values_close(got, want, rel, what, abs_tol=0.0, max_frac=MAX_DIFF_FRAC):
    """Float values equal except for a small fraction, each within `rel` (relative) + `abs_tol`."""
    got = np.asarray(got, dtype=np.float64).reshape(-1)
    want = np.asarray(want, dtype=np.float64).reshape(-1)
    diff = got != want
    both_nan = np.isnan(got) & np.isnan(want)
    diff &= ~both_nan
    n = int(diff.sum())
    if n == 0:
        return 0
    frac = n / got.size
    assert frac <= max_frac, f"{what}: {n} of {got.size} values differ ({frac:.2e} > {max_frac})"
    g, w = got[diff], want[diff]
    tol = rel * np.maximum(np.abs(g), np.abs(w)) + abs_tol
    worst = np.argmax(np.abs(g - w) - tol)
    assert np.all(np.abs(g - w) <= tol), f"{what}: {g[worst]} vs {w[worst]} beyond tolerance"
    return n


def qq_values(qq, qsf, T, sf_rows):
    """Dequantized q_c [T, 2048] from e4m3 codes and DeepGEMM-packed UE8M0 exponents."""
    codes = e4m3_to_f32(qq[:T * 2048]).reshape(T, 16, 128)
    words = qsf.reshape(4, sf_rows, 4)[:, :T, :]          # [kb >> 2][row][kb & 3]
    exps = words.transpose(1, 0, 2).reshape(T, 16).astype(np.int32)
    scale = np.ldexp(1.0, exps - 127).astype(np.float64)
    return codes * scale[:, :, None]


def latent_values(rows):
    """fp8_ds_mla rows [n, 656] -> kv_norm values [n, 512] and k_pe bits [n, 64]."""
    rows = np.ascontiguousarray(rows, dtype=np.uint8)
    codes = e4m3_to_f32(rows[:, :512]).reshape(-1, 4, 128).astype(np.float64)
    sc = rows[:, 512:528].copy().view(np.float32).astype(np.float64)
    return (codes * sc[:, :, None]).reshape(-1, 512), rows[:, 528:].copy().view(np.uint16)


def index_values(pages, slots):
    """Indexer keys of `slots` from a page pool -> values [n, 128]."""
    pages = pages.reshape(-1, 64 * 132)
    p, i = slots // 64, slots % 64
    keys = np.stack([pages[a, b * 128:(b + 1) * 128] for a, b in zip(p, i)])
    sc = np.stack([pages[a, 8192 + 4 * b:8196 + 4 * b].view(np.float32)[0] for a, b in zip(p, i)])
    return e4m3_to_f32(keys).astype(np.float64) * sc[:, None].astype(np.float64), sc


def assert_prep_close(got, want, case, full=True, what="prep"):
    """Append outputs of the device vs the C oracle (tolerances in the module docstring)."""
    T, sf_rows = case.T, case.sf_rows
    qg, qw = qq_values(got["qq"], got["qsf"], T, sf_rows), qq_values(want["qq"], want["qsf"], T, sf_rows)
    assert_values_close(qg, qw, E4M3_REL, f"{what}: q_c", abs_tol=0.0)
    slots = case.call.slot_mapping
    live = slots[slots >= 0]
    if case.kv_dtype == "fp8":
        rg = got["kv"].reshape(-1, 656)[live]
        rw = want["kv"].reshape(-1, 656)[live]
        vg, peg = latent_values(rg)
        vw, pew = latent_values(rw)
        assert_values_close(vg, vw, E4M3_REL, f"{what}: kv_norm", abs_tol=0.0)
        assert_equal(peg, pew, f"{what}: k_pe")
    else:
        rg = got["kv"].reshape(-1, 1152)[live].copy().view(np.uint16)
        rw = want["kv"].reshape(-1, 1152)[live].copy().view(np.uint16)
        assert_values_close(bf16_to_f32(rg[:, :512]), bf16_to_f32(rw[:, :512]), BF16_REL, f"{what}: kv_norm bf16")
        assert_equal(rg[:, 512:], rw[:, 512:], f"{what}: k_pe")
    if full:
        kg_, sg = index_values(got["idx"], live)
        kw_, sw = index_values(want["idx"], live)
        assert_values_close(kg_, kw_, E4M3_REL, f"{what}: indexer key")
        assert_values_close(sg, sw, 1.0, f"{what}: indexer scale")  # a power of two either side
