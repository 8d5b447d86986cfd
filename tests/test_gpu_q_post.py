"""glm_q_post (the q_pe rope into qmla's tail, the indexer query and its head weights) against the
reference kernel and the C oracle: bit-exact, on indexer and shared layers."""
import numpy as np
import pytest

from compare import assert_equal
from layer_case import LDB, q_post_case

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

def run_case(c, full, impl, cuda):
    import glmkv
    from oracle import ref
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    T = c["T"]
    qb, rope, pos, iw = t(c["qb"].view(np.int16)), t(c["rope"].view(np.int16)), t(c["pos"]), t(c["iw"].view(np.int16))
    qmla = torch.full((T * 64 * 576,), 0x1234, dtype=torch.int16, device=cuda)  # untouched outside the tails
    iq = torch.zeros(T * 32 * 128, dtype=torch.uint8, device=cuda)
    wout = torch.zeros(T * 32, dtype=torch.float32, device=cuda)
    if impl == "glmkv":
        if full:
            glmkv.q_post_full(qb, c["ldb"], rope, pos, qmla, iq, iw, wout, 1, T)
        else:
            glmkv.q_post_shared(qb, c["ldb"], rope, pos, qmla, 0, T)
    else:
        p = lambda x: x.data_ptr()
        ref.q_post(p(qb), c["ldb"], p(rope), p(pos), p(qmla), p(iq) if full else None, p(iw) if full else None,
                   p(wout) if full else None, int(full), T)
    torch.cuda.synchronize()
    return qmla.cpu().numpy().view(np.uint16), iq.cpu().numpy(), wout.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("full", [True, False])
@pytest.mark.parametrize("T", [1, 37, 512])
def test_q_post_vs_reference_and_oracle(cuda, ref, full, T):
    from oracle import cpu
    c = q_post_case(T, 100 + T)
    got = run_case(c, full, "glmkv", cuda)
    want = run_case(c, full, "reference", cuda)
    for g, w, name in zip(got, want, ("qmla", "iq", "wout")):
        assert_equal(g, w, f"q_post vs reference: {name}")
    qmla = np.full(T * 64 * 576, 0x1234, np.uint16)
    iq = np.zeros(T * 32 * 128, np.uint8)
    wout = np.zeros(T * 32, np.float32)
    cpu.q_post(c["qb"], c["ldb"], c["rope"], c["pos"], qmla, iq if full else None, c["iw"] if full else None,
               wout if full else None, full, T)
    for g, w, name in zip(got, (qmla, iq, wout.view(np.uint32)), ("qmla", "iq", "wout")):
        assert_equal(g, w, f"q_post vs oracle: {name}")


@pytest.mark.parametrize("full", [True, False])
def test_q_post_16384_rows_vs_reference(cuda, ref, full):
    c = q_post_case(16384, 7)
    for g, w, name in zip(run_case(c, full, "glmkv", cuda), run_case(c, full, "reference", cuda),
                          ("qmla", "iq", "wout")):
        assert_equal(g, w, f"16384 rows: {name}")


def test_q_post_wider_rows(cuda, ref):
    """qb rows wider than the 20,480 columns the op reads (ldb 20,488)."""
    c = q_post_case(64, 3, ldb=LDB + 8)
    for g, w, name in zip(run_case(c, True, "glmkv", cuda), run_case(c, True, "reference", cuda),
                          ("qmla", "iq", "wout")):
        assert_equal(g, w, f"ldb {LDB + 8}: {name}")
