"""ctypes wrapper of the reference's own glue kernels (``oracle/_ref/libglmref.so``). TEST INFRASTRUCTURE ONLY.

The library is kern-glm53 ``source/glm_glue.cu`` compiled unmodified for sm_100a (``oracle/build.py``)
with host launchers that use the manifest grids (``oracle/ref_launch.cu``). Arguments are raw device
addresses (ints) as in the reference's own launches, plus ``ctx`` where the manifest grid needs it and
the stream handle.
"""
import ctypes

from . import build as _build

_lib = None


class RefUnavailable(RuntimeError):
    pass


def available():
    return _build.REF_SO.exists()


def lib():
    global _lib
    if _lib is None:
        if not _build.REF_SO.exists() and _build.build_ref() is None:
            raise RefUnavailable(f"{_build.REF_SO} is missing: build it with `python oracle/build.py --ref-root "
                                 "<kern-glm53 checkout>`")
        _lib = ctypes.CDLL(str(_build.REF_SO))
        P, I = ctypes.c_void_p, ctypes.c_int
        _lib.ref_glm_plan.argtypes = [P, P, I, P, P, P, P, P, P, I, P]
        _lib.ref_glm_mla_prep.argtypes = [I, P, I, P, P, P, P, P, P, P, P, P, P, P, I, I, P]
        _lib.ref_glm_idx_gather.argtypes = [P, P, I, P, I, P, P, I, P]
        _lib.ref_glm_kv_dequant.argtypes = [P, P, I, P, I, P, I, P]
        _lib.ref_glm_topk_stream.argtypes = [P, P, P, P, I, P]
        _lib.ref_glm_topk_slots.argtypes = [P, P, I, P, P, P, I, P]
        _lib.ref_glm_q_post.argtypes = [P, I, P, P, P, P, P, P, I, I, P]
        _lib.ref_glm_add_rms_quant.argtypes = [P, P, P, P, P, P, I, I, P]
        _lib.ref_glm_quant.argtypes = [P, I, P, P, I, I, I, P]
    return _lib


def _check(rc, name):
    if rc != 0:
        raise RuntimeError(f"reference {name} launch failed with CUDA error {rc}")


def plan(cu, seq_lens, nseq, pos, ks, ke, klen, row_seq, zero, T, stream=0):
    _check(lib().ref_glm_plan(cu, seq_lens, nseq, pos, ks, ke, klen, row_seq, zero, T, stream), "glm_plan")


def mla_prep(fp8, x, lda, g_q, g_kv, rope, pos, slot, kv, idx, ik_w, ik_b, qq, qsf, sf_rows, T, stream=0):
    _check(lib().ref_glm_mla_prep(int(bool(fp8)), x, lda, g_q, g_kv, rope, pos, slot, kv, idx, ik_w, ik_b, qq, qsf,
                                  sf_rows, T, stream), "glm_mla_prep")


def idx_gather(idx, block_table, max_pages, seq_lens, nseq, kg, ksf, ctx, stream=0):
    _check(lib().ref_glm_idx_gather(idx, block_table, max_pages, seq_lens, nseq, kg, ksf, ctx, stream),
           "glm_idx_gather")


def kv_dequant(kv, block_table, max_pages, seq_lens, nseq, kvd, ctx, stream=0):
    _check(lib().ref_glm_kv_dequant(kv, block_table, max_pages, seq_lens, nseq, kvd, ctx, stream), "glm_kv_dequant")


def topk_stream(ind, ks, klen, tlen, T, stream=0):
    _check(lib().ref_glm_topk_stream(ind, ks, klen, tlen, T, stream), "glm_topk_stream")


def topk_slots(ind, block_table, max_pages, row_seq, klen, tlen, T, stream=0):
    _check(lib().ref_glm_topk_slots(ind, block_table, max_pages, row_seq, klen, tlen, T, stream), "glm_topk_slots")


def q_post(qb, ldb, rope, pos, qmla, iq, iw, wout, full, T, stream=0):
    _check(lib().ref_glm_q_post(qb, ldb, rope, pos, qmla, iq, iw, wout, int(bool(full)), T, stream), "glm_q_post")


def add_rms_quant(a, res, gamma, normed, q, sf, sf_rows, T, stream=0):
    _check(lib().ref_glm_add_rms_quant(a, res, gamma, normed, q, sf, sf_rows, T, stream), "glm_add_rms_quant")


def quant(x, ldx, q, sf, sf_rows, K, T, stream=0):
    _check(lib().ref_glm_quant(x, ldx, q, sf, sf_rows, K, T, stream), "glm_quant")
