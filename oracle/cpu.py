"""NumPy-facing wrapper of the C oracle (``glm_oracle.c``). TEST INFRASTRUCTURE ONLY.

Arrays are plain NumPy: bf16 tensors travel as ``uint16`` bit patterns, e4m3 as ``uint8``.
Each function mirrors one reference entry of kern-glm53 ``source/glm_glue.cu`` with the same argument
order (minus the stream); outputs are written in place like the kernels do.
"""
import ctypes
import numpy as np

from . import build as _build

_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(_build.build_oracle()))
        P = ctypes.c_void_p
        I = ctypes.c_int
        _lib.orc_plan.argtypes = [P, P, I, P, P, P, P, P, P, I]
        _lib.orc_mla_prep.argtypes = [I, P, I, P, P, P, P, P, P, P, P, P, P, P, I, I]
        _lib.orc_idx_gather.argtypes = [P, P, I, P, I, P, P]
        _lib.orc_kv_dequant.argtypes = [P, P, I, P, I, P]
        _lib.orc_topk_stream.argtypes = [P, P, P, P, I]
        _lib.orc_topk_slots.argtypes = [P, P, I, P, P, P, I]
        _lib.orc_q_post.argtypes = [P, I, P, P, P, P, P, P, I, I]
        _lib.orc_add_rms_quant.argtypes = [P, P, P, P, P, P, I, I]
        _lib.orc_quant.argtypes = [P, I, P, P, I, I, I]
        _lib.orc_bf16_from_f32.argtypes = [P, P, ctypes.c_long]
        _lib.orc_e4m3_from_f32.argtypes = [P, P, ctypes.c_long]
        _lib.orc_f32_from_e4m3.argtypes = [P, P, ctypes.c_long]
        _lib.orc_set_idx_fma.argtypes = [I]
        _lib.orc_get_idx_fma.restype = I
        _lib.orc_threads.restype = I
        _lib.orc_set_threads.argtypes = [I]
    return _lib


def _p(a, dtype=None):
    """Pointer of a C-contiguous array (or None for a null argument)."""
    if a is None:
        return None
    assert isinstance(a, np.ndarray) and a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    if dtype is not None:
        assert a.dtype == dtype, (a.dtype, dtype)
    return a.ctypes.data


def threads():
    return lib().orc_threads()


def set_threads(n):
    lib().orc_set_threads(int(n))


def set_idx_fma(flags):
    lib().orc_set_idx_fma(int(flags))


def plan(cu, seq_lens, nseq, pos, ks, ke, klen, row_seq, zero, T):
    lib().orc_plan(_p(cu, np.int64), _p(seq_lens, np.int32), nseq, _p(pos, np.int32), _p(ks, np.uint32),
                   _p(ke, np.uint32), _p(klen, np.int32), _p(row_seq, np.int32), _p(zero, np.int32), T)


def mla_prep(fp8, x, lda, g_q, g_kv, rope, pos, slot, kv, idx, ik_w, ik_b, qq, qsf, sf_rows, T):
    lib().orc_mla_prep(int(bool(fp8)), _p(x, np.uint16), lda, _p(g_q, np.uint16), _p(g_kv, np.uint16),
                       _p(rope, np.uint16), _p(pos, np.int32), _p(slot, np.int64), _p(kv, np.uint8), _p(idx, np.uint8),
                       _p(ik_w, np.uint16), _p(ik_b, np.uint16), _p(qq, np.uint8), _p(qsf, np.uint8), sf_rows, T)


def idx_gather(idx, block_table, max_pages, seq_lens, nseq, kg, ksf):
    lib().orc_idx_gather(_p(idx, np.uint8), _p(block_table, np.int32), max_pages, _p(seq_lens, np.int32), nseq,
                         _p(kg, np.uint8), _p(ksf, np.float32))


def kv_dequant(kv, block_table, max_pages, seq_lens, nseq, kvd):
    lib().orc_kv_dequant(_p(kv, np.uint8), _p(block_table, np.int32), max_pages, _p(seq_lens, np.int32), nseq,
                         _p(kvd, np.uint16))


def topk_stream(ind, ks, klen, tlen, T):
    lib().orc_topk_stream(_p(ind, np.int32), _p(ks, np.uint32), _p(klen, np.int32), _p(tlen, np.int32), T)


def topk_slots(ind, block_table, max_pages, row_seq, klen, tlen, T):
    lib().orc_topk_slots(_p(ind, np.int32), _p(block_table, np.int32), max_pages, _p(row_seq, np.int32),
                         _p(klen, np.int32), _p(tlen, np.int32), T)


def bf16_from_f32(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(x.shape, np.uint16)
    lib().orc_bf16_from_f32(_p(x), _p(y), x.size)
    return y


def e4m3_from_f32(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(x.shape, np.uint8)
    lib().orc_e4m3_from_f32(_p(x), _p(y), x.size)
    return y


def f32_from_e4m3(x):
    x = np.ascontiguousarray(x, dtype=np.uint8)
    y = np.empty(x.shape, np.float32)
    lib().orc_f32_from_e4m3(_p(x), _p(y), x.size)
    return y


def q_post(qb, ldb, rope, pos, qmla, iq, iw, wout, full, T):
    lib().orc_q_post(_p(qb, np.uint16), ldb, _p(rope, np.uint16), _p(pos, np.int32), _p(qmla, np.uint16),
                     _p(iq, np.uint8), _p(iw, np.uint16), _p(wout, np.float32), int(bool(full)), T)


def add_rms_quant(a, res, gamma, normed, q, sf, sf_rows, T):
    lib().orc_add_rms_quant(_p(a, np.uint16), _p(res, np.uint16), _p(gamma, np.uint16), _p(normed, np.uint16),
                            _p(q, np.uint8), _p(sf, np.uint8), sf_rows, T)


def quant(x, ldx, q, sf, sf_rows, K, T):
    lib().orc_quant(_p(x, np.uint16), ldx, _p(q, np.uint8), _p(sf, np.uint8), sf_rows, K, T)
