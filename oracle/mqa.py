"""The indexer's fp8 MQA logits, restated in NumPy. TEST INFRASTRUCTURE ONLY. Parity unpinned: the
reference's own kernel for this (DeepGEMM) is absent, so no reference output exists to pin it to.

kern-glm53 scores each fresh row against every key of its sequence with DeepGEMM's sm100 fp8 MQA
logits (scripts/glm_ops.py:104-134: ``MQA_ENTRY``, launched on the gathered ``kg`` / ``ksf`` stream
that ``glm_idx_gather`` writes). DeepGEMM is an empty submodule in kern-glm53 (pinned at ``ab69f76b``,
kernels.toml:9-17), so this module restates its published definition, the one DeepGEMM's own tests
check ``fp8_mqa_logits`` against:

    logits[r, p] = sum_h w[r, h] * relu( sum_d q[r, h, d] * k[p, d] * s[p] )

for every key position p of row r's sequence below klen[r] (``ke - ks`` in the compressed layout:
row r's logits at [r][0, ke - ks), glm_ops.py:104-105). q is the e4m3 indexer query [R, 32, 128] that
``glm_q_post`` writes (its UE8M0 scale is folded into w, glm_glue.cu:340-347), k the e4m3 indexer key
and s its f32 scale from the page-blocked indexer cache (page = block_table[seq][p / 64], row p % 64;
keys at row * 128, scales at 8192 + 4 * row).

Here the key rows are read straight from the cache pages -- the gather-free input format -- which
gives the same numbers as reading the gathered stream. Each dot product is exact in float64 (128
products of two e4m3 values, 8 significant bits each, exponents within 2^-18 .. 2^16), so the only
rounding is the final float64 sum; a device result computed in f32 is compared with a tolerance
relative to ``magnitude`` (the same sum with |.| everywhere).
"""
import numpy as np

PAGE, ID, IH, IDX_PAGE = 64, 128, 32, 64 * 132


def e4m3_table():
    """f32 value of every e4m3 code (S.EEEE.MMM, bias 7; 0x7F / 0xFF are NaN)."""
    t = np.zeros(256, np.float64)
    for c in range(256):
        s = -1.0 if c & 0x80 else 1.0
        e, m = (c >> 3) & 0xF, c & 7
        if e == 0xF and m == 7:
            t[c] = np.nan
        elif e == 0:
            t[c] = s * m * 2.0 ** -9
        else:
            t[c] = s * (1 + m / 8) * 2.0 ** (e - 7)
    return t


E4M3 = e4m3_table()


def keys_of(idx_pool, block_table, max_pages, seq, n):
    """The first n indexer keys of sequence `seq` (as float64 [n, 128]) and their f32 scales."""
    pages = idx_pool.reshape(-1, IDX_PAGE)
    bt = block_table.reshape(-1, max_pages)[seq]
    p = np.arange(n)
    page, row = bt[p // PAGE], p % PAGE
    codes = pages[page[:, None], row[:, None] * ID + np.arange(ID)[None, :]]
    scale_bytes = pages[page[:, None], PAGE * ID + 4 * row[:, None] + np.arange(4)[None, :]]
    scales = np.ascontiguousarray(scale_bytes).view(np.float32).reshape(n)
    return E4M3[codes], scales.astype(np.float64)


def mqa_logits_paged(iq, idx_pool, block_table, max_pages, row_seq, klen, w):
    """Per row r: (logits [klen[r]], magnitude [klen[r]]) as float64, in a list."""
    R = len(row_seq)
    q = E4M3[iq.reshape(R, IH, ID)]
    w = np.asarray(w, np.float64).reshape(R, IH)
    out = []
    for s in np.unique(row_seq):
        rows = np.nonzero(row_seq == s)[0]
        n = int(klen[rows].max())
        k, sc = keys_of(idx_pool, block_table, max_pages, int(s), n)
        dots = np.einsum("rhd,pd->rhp", q[rows], k)                       # exact
        mags = np.einsum("rhd,pd->rhp", np.abs(q[rows]), np.abs(k))
        for i, r in enumerate(rows):
            m = int(klen[r])
            lg = (w[r][:, None] * np.maximum(dots[i, :, :m] * sc[None, :m], 0)).sum(0)
            mg = (np.abs(w[r])[:, None] * mags[i, :, :m] * sc[None, :m]).sum(0)
            out.append((r, lg, mg))
    out.sort(key=lambda t: t[0])
    return [(lg, mg) for _, lg, mg in out]


def flops(klen):
    """Multiply-adds of the dot products, as FLOPs (2 a multiply-add): 32 heads x 128 dims a key."""
    return int(np.sum(np.asarray(klen, np.int64))) * IH * ID * 2
