"""glm_add_rms_quant (residual add + RMSNorm + quant) and glm_quant against the reference kernels
(bit-exact) and the C oracle (glm_quant bit-exact; the norm within the rsqrtf tolerance)."""
import numpy as np
import pytest

from compare import E4M3_REL, BF16_REL, assert_equal, assert_values_close, bf16_to_f32, e4m3_to_f32
from layer_case import norm_case as _inputs, quant_case

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
H = 6144


def _run(impl, a, res, gamma, T, want_normed, want_q, cuda):
    import glmkv
    from oracle import ref
    t = lambda x: None if x is None else torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).to(cuda)
    da, dres, dg = t(a), t(res), t(gamma)
    normed = torch.zeros(T * H, dtype=torch.int16, device=cuda) if want_normed else None
    q = torch.zeros(T * H, dtype=torch.uint8, device=cuda) if want_q else None
    sf = torch.zeros((H // 512) * T * 4, dtype=torch.uint8, device=cuda) if want_q else None
    if impl == "glmkv":
        glmkv.add_rms_quant(da, dres, dg, normed, q, sf, T, T)
    else:
        p = lambda x: None if x is None else x.data_ptr()
        ref.add_rms_quant(p(da), p(dres), p(dg), p(normed), p(q), p(sf), T, T)
    torch.cuda.synchronize()
    g = lambda x: None if x is None else x.cpu().numpy()
    return {"res": g(dres).view(np.uint16), "normed": g(normed), "q": g(q), "sf": g(sf)}


CASES = [(1, True, True, True), (37, True, True, True), (512, True, True, True), (512, False, True, True),
         (64, True, True, False), (64, True, False, True)]


@pytest.mark.parametrize("T,with_a,want_normed,want_q", CASES)
def test_add_rms_quant_vs_reference_and_oracle(cuda, ref, T, with_a, want_normed, want_q):
    from oracle import cpu
    a, res, gamma = _inputs(T, 1000 + T + 7 * with_a, with_a)
    got = _run("glmkv", a, res, gamma, T, want_normed, want_q, cuda)
    want = _run("reference", a, res, gamma, T, want_normed, want_q, cuda)
    for k in got:
        if got[k] is not None:
            assert_equal(got[k].view(np.uint8), want[k].view(np.uint8), f"add_rms_quant vs reference: {k}")
    r2 = res.copy()
    normed = np.zeros(T * H, np.uint16) if want_normed else None
    q = np.zeros(T * H, np.uint8) if want_q else None
    sf = np.zeros((H // 512) * T * 4, np.uint8) if want_q else None
    cpu.add_rms_quant(a, r2, gamma, normed, q, sf, T, T)
    assert_equal(got["res"].reshape(-1), r2.reshape(-1), "add_rms_quant vs oracle: res")  # the add has no rsqrt
    if want_normed:
        assert_values_close(bf16_to_f32(got["normed"].view(np.uint16)), bf16_to_f32(normed), BF16_REL,
                            "add_rms_quant vs oracle: normed")
    if want_q:
        def vals(qq, ss):
            e = ss.reshape(H // 512, T, 4).transpose(1, 0, 2).reshape(T, H // 128).astype(np.int32)
            return e4m3_to_f32(qq).reshape(T, H // 128, 128) * np.ldexp(1.0, e - 127)[:, :, None]
        assert_values_close(vals(got["q"], got["sf"]), vals(q, sf), E4M3_REL, "add_rms_quant vs oracle: q")


def test_add_rms_quant_16384_rows_vs_reference(cuda, ref):
    a, res, gamma = _inputs(16384, 5)
    got = _run("glmkv", a, res, gamma, 16384, True, True, cuda)
    want = _run("reference", a, res, gamma, 16384, True, True, cuda)
    for k in got:
        assert_equal(got[k].view(np.uint8), want[k].view(np.uint8), f"16384 rows: {k}")


@pytest.mark.parametrize("T,K,ldx", [(1, 128, 128), (37, 640, 648), (512, 16384, 16384), (16384, 16384, 16384)])
def test_quant_vs_reference_and_oracle(cuda, ref, T, K, ldx):
    import glmkv
    from glmkv import workload as W
    from oracle import cpu
    x = quant_case(T, K, ldx)
    dx = torch.from_numpy(x.view(np.int16)).to(cuda)
    sf_words = (K + 511) // 512
    outs = []
    for impl in ("glmkv", "reference"):
        q = torch.zeros(T * K, dtype=torch.uint8, device=cuda)
        sf = torch.zeros(sf_words * T * 4, dtype=torch.uint8, device=cuda)
        if impl == "glmkv":
            glmkv.quant_o(dx, ldx, q, sf, T, K, T)
        else:
            ref.quant(dx.data_ptr(), ldx, q.data_ptr(), sf.data_ptr(), T, K, T)
        torch.cuda.synchronize()
        outs.append((q.cpu().numpy(), sf.cpu().numpy()))
    assert_equal(outs[0][0], outs[1][0], "quant vs reference: q")
    assert_equal(outs[0][1], outs[1][1], "quant vs reference: sf")
    if T <= 512:
        q = np.zeros(T * K, np.uint8)
        sf = np.zeros(sf_words * T * 4, np.uint8)
        cpu.quant(x, ldx, q, sf, T, K, T)
        assert_equal(outs[0][0], q, "quant vs oracle: q")
        assert_equal(outs[0][1], sf, "quant vs oracle: sf")
