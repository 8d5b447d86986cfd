"""The KV-cache ops under the names and argument orders of the kern-glm53 manifest (scripts/gen.py).

Every op takes device buffers as CUDA ``torch.Tensor`` (or raw device addresses as ``int``) followed
by the op's scalars, exactly in the manifest's parameter order, and enqueues one kernel of
``libglmkv.so`` on ``stream`` (default: torch's current stream). PyTorch only owns the memory.

    op               manifest params (gen.py)                              kernel
    plan             cu, seq_lens, nseq, pos, ks, ke, klen, row_seq,      glm_plan
                     zero, T                                  (95-98)
    mla_prep_full    x, lda, g_q, g_kv, rope, pos, slot, kv, idx, ik_w,   glm_mla_prep_fp8 / glm_mla_prep
                     ik_b, qq, qsf, sf_rows, T              (172-176)
    mla_prep_shared  the same without idx, ik_w, ik_b (nulled, 177)       glm_mla_prep_fp8 / glm_mla_prep
    idx_gather       idx, block_table, max_pages, seq_lens, nseq, kg, ksf glm_idx_gather
                                                            (124-126)
    kv_dequant       kv, block_table, max_pages, seq_lens, nseq, kvd      glm_kv_dequant
                                                            (133-135)
    topk_stream      ind, ks, klen, tlen, T                 (130-132)     glm_topk_stream
    topk_slots       ind, block_table, max_pages, row_seq, klen, tlen, T  glm_topk_slots
                                                            (127-129)
    q_post_full      qb, ldb, rope, pos, qmla, iq, iw, wout, full, T       glm_q_post
                                                            (117-119)
    q_post_shared    the same without iq, iw, wout (nulled, 120-123)       glm_q_post
    add_rms_quant    a, res, gamma, normed, q, sf, sf_rows, T (168-170)    glm_add_rms_quant
    rms_quant        the same without a (nulled, 171)                      glm_add_rms_quant
    head_norm        the same without q, sf (nulled, 156-158)              glm_add_rms_quant
    quant_o          x, ldx, q, sf, sf_rows, K, T         (103-105)        glm_quant
    mark_rows        ind, ks, ke, T, mask, mask_words: the bitmap of the    glm_mark_rows
                     stream rows the picks name (no manifest op: feeds
                     kv_dequant_marked)
    topk_stream_mark ind, ks, klen, tlen, T, ke, mask, mask_words:   glm_topk_stream_mark
                     topk_stream and mark_rows in one pass (replaces
                     topk_stream where the marked lift is used)
    kv_dequant_marked kv, block_table, max_pages, seq_lens, nseq, mask,  glm_kv_dequant_marked
                     kvd: the lift of the marked rows only
    mqa_logits_paged iq, idx, n_pages, block_table, max_pages, row_seq,  glm_mqa_logits_paged
                     klen, w, logits, stride, R: the indexer's MQA logits
                     from the cache pages (replaces idx_gather + the MQA
                     launch of indexer.<j>, glm_ops.py:104-134)

Errors (null or misaligned buffers, sizes out of range, a failed launch) raise ``GlmKvError``.
"""
import torch

from . import _lib

_DTYPES = {
    "i64": (torch.int64,),
    "i32": (torch.int32,),
    "u32": (torch.int32, torch.uint32),
    "bf16": (torch.bfloat16, torch.int16, torch.uint16),
    "u8": (torch.uint8, torch.int8, torch.float8_e4m3fn),
    "f32": (torch.float32,),
    "u64": (torch.int64, torch.uint64),
}


def _ptr(a, kind, name):
    """A device address from a CUDA tensor (dtype-checked), an int, or None (null)."""
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if not isinstance(a, torch.Tensor):
        raise TypeError(f"{name}: expected a CUDA tensor or a device address, got {type(a).__name__}")
    if not a.is_cuda:
        raise ValueError(f"{name}: tensor is on {a.device}, the kernels need device memory")
    if a.dtype not in _DTYPES[kind]:
        raise TypeError(f"{name}: dtype {a.dtype} where {kind} is expected")
    if not a.is_contiguous():
        raise ValueError(f"{name}: tensor must be contiguous")
    return a.data_ptr()


def _stream(stream):
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def plan(cu, seq_lens, nseq, pos, ks, ke, klen, row_seq, zero, T, stream=None):
    _lib.call("glmkv_plan", _ptr(cu, "i64", "cu"), _ptr(seq_lens, "i32", "seq_lens"), int(nseq),
              _ptr(pos, "i32", "pos"), _ptr(ks, "u32", "ks"), _ptr(ke, "u32", "ke"), _ptr(klen, "i32", "klen"),
              _ptr(row_seq, "i32", "row_seq"), _ptr(zero, "i32", "zero"), int(T), _stream(stream))


def _prep(fp8, x, lda, g_q, g_kv, rope, pos, slot, kv, idx, ik_w, ik_b, qq, qsf, sf_rows, T, stream):
    name = "glmkv_mla_prep_fp8" if fp8 else "glmkv_mla_prep"
    _lib.call(name, _ptr(x, "bf16", "x"), int(lda), _ptr(g_q, "bf16", "g_q"), _ptr(g_kv, "bf16", "g_kv"),
              _ptr(rope, "bf16", "rope"), _ptr(pos, "i32", "pos"), _ptr(slot, "i64", "slot"), _ptr(kv, "u8", "kv"),
              _ptr(idx, "u8", "idx"), _ptr(ik_w, "bf16", "ik_w"), _ptr(ik_b, "bf16", "ik_b"), _ptr(qq, "u8", "qq"),
              _ptr(qsf, "u8", "qsf"), int(sf_rows), int(T), _stream(stream))


def mla_prep_full(x, lda, g_q, g_kv, rope, pos, slot, kv, idx, ik_w, ik_b, qq, qsf, sf_rows, T, *, kv_dtype="fp8",
                  stream=None):
    """The append of an indexer layer: latent row and indexer key (op `mla_prep_full`)."""
    _prep(kv_dtype == "fp8", x, lda, g_q, g_kv, rope, pos, slot, kv, idx, ik_w, ik_b, qq, qsf, sf_rows, T, stream)


def mla_prep_shared(x, lda, g_q, g_kv, rope, pos, slot, kv, qq, qsf, sf_rows, T, *, kv_dtype="fp8", stream=None):
    """The append of a shared layer: latent row only (op `mla_prep_shared`, idx / ik_w / ik_b null)."""
    _prep(kv_dtype == "fp8", x, lda, g_q, g_kv, rope, pos, slot, kv, None, None, None, qq, qsf, sf_rows, T, stream)


def idx_gather(idx, block_table, max_pages, seq_lens, nseq, kg, ksf, stream=None):
    _lib.call("glmkv_idx_gather", _ptr(idx, "u8", "idx"), _ptr(block_table, "i32", "block_table"), int(max_pages),
              _ptr(seq_lens, "i32", "seq_lens"), int(nseq), _ptr(kg, "u8", "kg"), _ptr(ksf, "f32", "ksf"),
              _stream(stream))


def kv_dequant(kv, block_table, max_pages, seq_lens, nseq, kvd, stream=None):
    _lib.call("glmkv_kv_dequant", _ptr(kv, "u8", "kv"), _ptr(block_table, "i32", "block_table"), int(max_pages),
              _ptr(seq_lens, "i32", "seq_lens"), int(nseq), _ptr(kvd, "bf16", "kvd"), _stream(stream))


def mark_rows(ind, ks, ke, T, mask, mask_words, stream=None):
    """The bitmap of the stream rows the picks name (bit p % 64 of word p // 64), cleared first."""
    _lib.call("glmkv_mark_rows", _ptr(ind, "i32", "ind"), _ptr(ks, "u32", "ks"), _ptr(ke, "u32", "ke"), int(T),
              _ptr(mask, "u64", "mask"), int(mask_words), _stream(stream))


def topk_stream_mark(ind, ks, klen, tlen, T, ke, mask, mask_words, stream=None):
    """topk_stream (ind sequence-relative in, stream rows out, in place; tlen) and mark_rows of the
    result, in one pass over the picks."""
    _lib.call("glmkv_topk_stream_mark", _ptr(ind, "i32", "ind"), _ptr(ks, "u32", "ks"), _ptr(klen, "i32", "klen"),
              _ptr(tlen, "i32", "tlen"), int(T), _ptr(ke, "u32", "ke"), _ptr(mask, "u64", "mask"), int(mask_words),
              _stream(stream))


def kv_dequant_marked(kv, block_table, max_pages, seq_lens, nseq, mask, kvd, stream=None):
    """kv_dequant of the rows `mask` marks only; the other rows of kvd are not written."""
    _lib.call("glmkv_kv_dequant_marked", _ptr(kv, "u8", "kv"), _ptr(block_table, "i32", "block_table"),
              int(max_pages), _ptr(seq_lens, "i32", "seq_lens"), int(nseq), _ptr(mask, "u64", "mask"),
              _ptr(kvd, "bf16", "kvd"), _stream(stream))


def topk_stream(ind, ks, klen, tlen, T, stream=None):
    _lib.call("glmkv_topk_stream", _ptr(ind, "i32", "ind"), _ptr(ks, "u32", "ks"), _ptr(klen, "i32", "klen"),
              _ptr(tlen, "i32", "tlen"), int(T), _stream(stream))


def topk_slots(ind, block_table, max_pages, row_seq, klen, tlen, T, stream=None):
    _lib.call("glmkv_topk_slots", _ptr(ind, "i32", "ind"), _ptr(block_table, "i32", "block_table"), int(max_pages),
              _ptr(row_seq, "i32", "row_seq"), _ptr(klen, "i32", "klen"), _ptr(tlen, "i32", "tlen"), int(T),
              _stream(stream))


def q_post_full(qb, ldb, rope, pos, qmla, iq, iw, wout, full, T, stream=None):
    """The q_pe rope and, when `full`, the indexer query and head weights (op `q_post_full`)."""
    _lib.call("glmkv_q_post", _ptr(qb, "bf16", "qb"), int(ldb), _ptr(rope, "bf16", "rope"), _ptr(pos, "i32", "pos"),
              _ptr(qmla, "bf16", "qmla"), _ptr(iq, "u8", "iq"), _ptr(iw, "bf16", "iw"), _ptr(wout, "f32", "wout"),
              int(full), int(T), _stream(stream))


def q_post_shared(qb, ldb, rope, pos, qmla, full, T, stream=None):
    """The q_pe rope of a shared layer (op `q_post_shared`, iq / iw / wout null)."""
    _lib.call("glmkv_q_post", _ptr(qb, "bf16", "qb"), int(ldb), _ptr(rope, "bf16", "rope"), _ptr(pos, "i32", "pos"),
              _ptr(qmla, "bf16", "qmla"), None, None, None, int(full), int(T), _stream(stream))


def add_rms_quant(a, res, gamma, normed, q, sf, sf_rows, T, stream=None):
    """res = bf16(a + res); normed = RMSNorm(res) * gamma; e4m3 per 128 columns (op `add_rms_quant`)."""
    _lib.call("glmkv_add_rms_quant", _ptr(a, "bf16", "a"), _ptr(res, "bf16", "res"), _ptr(gamma, "bf16", "gamma"),
              _ptr(normed, "bf16", "normed"), _ptr(q, "u8", "q"), _ptr(sf, "u8", "sf"), int(sf_rows), int(T),
              _stream(stream))


def rms_quant(res, gamma, normed, q, sf, sf_rows, T, stream=None):
    """The first layer's norm: res is already the stream (op `rms_quant`, a null)."""
    add_rms_quant(None, res, gamma, normed, q, sf, sf_rows, T, stream)


def head_norm(a, res, gamma, normed, sf_rows, T, stream=None):
    """The final norm of each sequence's last row, no quant (op `head_norm`, q and sf null)."""
    add_rms_quant(a, res, gamma, normed, None, None, sf_rows, T, stream)


def quant_o(x, ldx, q, sf, sf_rows, K, T, stream=None):
    """x [T, K] e4m3 per 128 columns with packed UE8M0 scales (op `quant_o`)."""
    _lib.call("glmkv_quant", _ptr(x, "bf16", "x"), int(ldx), _ptr(q, "u8", "q"), _ptr(sf, "u8", "sf"), int(sf_rows),
              int(K), int(T), _stream(stream))


def mqa_logits_paged(iq, idx, n_pages, block_table, max_pages, row_seq, klen, w, logits, stride, R, stream=None):
    """The indexer's fp8 MQA logits read from the indexer cache pages, on the tensor cores
    (op `mqa_logits_paged`): logits[r, p] for p < klen[r], row r's sequence row_seq[r]."""
    _lib.call("glmkv_mqa_logits_paged", _ptr(iq, "u8", "iq"), _ptr(idx, "u8", "idx"), int(n_pages),
              _ptr(block_table, "i32", "block_table"), int(max_pages), _ptr(row_seq, "i32", "row_seq"),
              _ptr(klen, "i32", "klen"), _ptr(w, "f32", "w"), _ptr(logits, "f32", "logits"), int(stride), int(R),
              _stream(stream))
