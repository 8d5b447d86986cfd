"""Algorithmic HBM bytes of each cache op: what the op must read and write at minimum, per launch.

The roofline of every op on this path is HBM bandwidth (no op does more than a few f32 operations a
byte). Units: a *fresh row* is one of the call's T new tokens; a *stream token* is one of the ctx
tokens (prefix + fresh) of the call's sequences.

    op                      unit           read                          write                     total
    kv_dequant              stream token   656 (fp8 row)                 1152 (bf16 row)           1808
    idx_gather              stream token   132 (key + scale)             132                       264
    mla_prep_fp8, full      fresh row      5504 x + 128 rope + 12        2048 qq + 16 qsf + 656    8496
                                           (pos, slot)                   kv + 132 idx
    mla_prep_fp8, shared    fresh row      5248 x + 128 + 12             2048 + 16 + 656           8108
    mla_prep (bf16 row)     fresh row      as above                      kv 1152 instead of 656    +496
    topk_stream/topk_slots  fresh row      8192 ind + 8 (ks/row, klen)   8192 ind + 4 tlen         16396
    plan                    fresh row      (cu, seq_lens: per call)      24 (six i32 / u32)        24

The next rows, around the path:

    q_post, indexer layer   fresh row      8192 q_pe + 8192 index query  8192 qmla tails + 4096    28996
                                           + 128 rope + 4 + 64 iw        iq + 128 wout
    q_post, shared layer    fresh row      8192 + 128 + 4                8192                      16516
    add_rms_quant           row            12288 a + 12288 res           12288 res + 12288 normed  55344
                                                                         + 6144 q + 48 sf
    rms_quant (no a)        row            12288 res                     12288 + 6144 + 48         30768
    quant (K columns)       row            2K                            K + K / 128               3K + K/128
"""
QL, KVL, ROPE, ID, TOPK = 2048, 512, 64, 128, 2048


def kv_dequant(ctx):
    return 1808 * ctx


def idx_gather(ctx):
    return 264 * ctx


def mla_prep(T, full=True, kv_dtype="fp8"):
    x = 2 * (QL + KVL + ROPE + (ID if full else 0))
    read = x + 2 * ROPE + 4 + 8
    write = QL + 16 + (656 if kv_dtype == "fp8" else 1152) + ((ID + 4) if full else 0)
    return (read + write) * T


def topk(T):
    return 16396 * T


def plan(T, nseq):
    return 24 * T + 12 * nseq + 8


def layer(T, ctx, full, kv_dtype="fp8"):
    """One layer's cache path as the manifest runs it (prep, [gather, row plan], dequant)."""
    b = mla_prep(T, full, kv_dtype)
    if full:
        b += idx_gather(ctx) + topk(T)
    if kv_dtype == "fp8":
        b += kv_dequant(ctx)
    return b


def q_post(T, full=True):
    return (28996 if full else 16516) * T


def add_rms_quant(T, with_a=True, normed=True, quant=True):
    H = 6144
    read = 2 * H * (2 if with_a else 1)
    write = (2 * H if with_a else 0) + (2 * H if normed else 0) + ((H + H // 128) if quant else 0)
    return (read + write) * T


def quant(T, K):
    return (3 * K + K // 128) * T
