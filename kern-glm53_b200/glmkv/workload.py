"""Seeded synthetic calls for the KV-cache path (NumPy), in the shapes and value distributions of the
reference's benchmark configurations. No public dataset is involved: every array comes from
``numpy.random.default_rng(seed)``.

A *call* is one packed prefill call as kern-glm53 builds it (scripts/kern_logits.py:61-88): up to 16
sequences, each with a prefix already cached and a fresh chunk appended by this call; the fresh
rows are packed back to back (``cu_seqlens``), ``seq_lens`` are prefix + fresh, pages are 64 tokens
and ``slot = page * 64 + offset`` through the block table (kern_logits.py:68, 78-81).

Configurations (cfg0 .. cfg4):
  cfg0  2 sequences: prefixes 1024 and 3072, 512 fresh rows each.
  cfg1  16 sequences, 16384 fresh rows split by Dirichlet(1) (>= 1 each, largest remainder), prefixes
        uniform in [0, 32768].
  cfg2  1 sequence: prefix 1,032,192 + 16384 fresh (2^20 tokens).
  cfg3  a layer's call of the 78-layer workload: 16 sequences, prefixes drawn from {0, 2K, 64K, 256K},
        fresh split as cfg1; redrawn until the stream is at most 2^20 tokens.
  cfg4  ragged edges: sequences of 1, 63, 64, 65, 2047, 2048 and 2049 tokens with empty prefixes,
        all-zero kv_a tiles; run with the bf16 latent cache.
"""
from dataclasses import dataclass, field

import numpy as np

PAGE = 64
QL, KVL, ROPE, ID = 2048, 512, 64, 128
NA_FULL = QL + KVL + ROPE + ID  # 2752: [q_a | kv_a | k_pe | wk]
TOPK = 2048
KV_ROW = {"fp8": 656, "bf16": 1152}
IDX_ROW = ID + 4
MAX_CTX = 1 << 20
THETA = 8e6  # GLM's rope base (kern-glm53 scripts/gen.py:259)
CFG3_PREFIXES = (0, 2048, 65536, 262144)


def bf16_bits(x):
    """float32 -> bf16 bit patterns (uint16), round to nearest even."""
    u = np.array(x, dtype=np.float32, copy=True).view(np.uint32)
    lsb = (u >> 16) & np.uint32(1)
    u += np.uint32(0x7FFF)
    u += lsb
    u >>= np.uint32(16)
    return u.astype(np.uint16)


def bf16_value(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


@dataclass
class Call:
    """The per-call metadata of one packed prefill call."""
    prefix: np.ndarray      # i32 [S]
    fresh: np.ndarray       # i32 [S]
    seq_lens: np.ndarray    # i32 [S] = prefix + fresh
    cu: np.ndarray          # i64 [S + 1], fresh-row prefix sums
    block_table: np.ndarray  # i32 [S, max_pages], -1 past a sequence's pages
    slot_mapping: np.ndarray  # i64 [T]
    n_pages: int            # physical pages the pool needs (page numbers 0 .. n_pages - 1)
    name: str = ""
    seed: int = 0
    extra: dict = field(default_factory=dict)

    @property
    def nseq(self):
        return int(len(self.seq_lens))

    @property
    def T(self):
        return int(self.cu[-1])

    @property
    def ctx(self):
        return int(self.seq_lens.sum())

    @property
    def max_pages(self):
        return int(self.block_table.shape[1])

    @property
    def stream_pages(self):
        return int(((self.seq_lens + PAGE - 1) // PAGE).sum())


def make_call(prefix, fresh, rng, max_pages=None, spare_pages=0, name="", seed=0):
    """A call over sequences (prefix[s], fresh[s]) with a seeded random permutation of physical pages."""
    prefix = np.asarray(prefix, dtype=np.int64)
    fresh = np.asarray(fresh, dtype=np.int64)
    lens = prefix + fresh
    pages = (lens + PAGE - 1) // PAGE
    total = int(pages.sum())
    max_pages = int(max_pages or max(1, int(pages.max())))
    assert max_pages >= pages.max()
    n_pages = total + int(spare_pages)
    perm = rng.permutation(n_pages)[:total].astype(np.int32)
    bt = np.full((len(lens), max_pages), -1, dtype=np.int32)
    o = 0
    for s, np_ in enumerate(pages):
        bt[s, :np_] = perm[o:o + np_]
        o += np_
    cu = np.zeros(len(lens) + 1, dtype=np.int64)
    cu[1:] = np.cumsum(fresh)
    slots = []
    for s in range(len(lens)):
        p = np.arange(prefix[s], lens[s], dtype=np.int64)
        slots.append(bt[s, p // PAGE].astype(np.int64) * PAGE + p % PAGE)
    slot = np.concatenate(slots) if slots else np.zeros(0, np.int64)
    return Call(prefix.astype(np.int32), fresh.astype(np.int32), lens.astype(np.int32), cu, bt, slot, n_pages,
                name=name, seed=seed)


def dirichlet_split(rng, total, parts):
    """`total` rows over `parts` sequences, >= 1 each, Dirichlet(1) weights, largest-remainder rounding."""
    w = rng.dirichlet(np.ones(parts))
    raw = w * (total - parts)
    base = np.floor(raw).astype(np.int64)
    left = (total - parts) - int(base.sum())
    order = np.argsort(-(raw - base), kind="stable")
    base[order[:left]] += 1
    return base + 1


def config(name, seed=0):
    """The call of configuration `name` ('cfg0' .. 'cfg4', or 'cfg1-bf16')."""
    rng = np.random.default_rng(seed)
    if name == "cfg0":
        return make_call([1024, 3072], [512, 512], rng, name=name, seed=seed)
    if name in ("cfg1", "cfg1-bf16"):
        fresh = dirichlet_split(rng, 16384, 16)
        prefix = rng.integers(0, 32768, size=16, endpoint=True)
        return make_call(prefix, fresh, rng, max_pages=MAX_CTX // PAGE, name=name, seed=seed)
    if name == "cfg2":
        return make_call([MAX_CTX - 16384], [16384], rng, max_pages=MAX_CTX // PAGE, name=name, seed=seed)
    if name == "cfg3":
        for draw in range(10000):
            fresh = dirichlet_split(rng, 16384, 16)
            prefix = rng.choice(CFG3_PREFIXES, size=16)
            if int((prefix + fresh).sum()) <= MAX_CTX:
                c = make_call(prefix, fresh, rng, max_pages=MAX_CTX // PAGE, name=name, seed=seed)
                c.extra["draws"] = draw + 1
                return c
        raise RuntimeError("no cfg3 draw fits 2^20 tokens")
    if name == "cfg4":
        lens = [1, 63, 64, 65, 2047, 2048, 2049]
        return make_call([0] * len(lens), lens, rng, name=name, seed=seed)
    raise KeyError(name)


# ------------------------------------------------------------------------------------------- tensors

@dataclass
class Weights:
    g_q: np.ndarray   # bf16 bits [2048]
    g_kv: np.ndarray  # bf16 bits [512]
    ik_w: np.ndarray  # bf16 bits [128]
    ik_b: np.ndarray  # bf16 bits [128]


def weights(rng):
    """Per-layer norm weights: gammas U(0.5, 1.5), LayerNorm bias N(0, 0.1)."""
    return Weights(bf16_bits(rng.uniform(0.5, 1.5, QL)), bf16_bits(rng.uniform(0.5, 1.5, KVL)),
                   bf16_bits(rng.uniform(0.5, 1.5, ID)), bf16_bits(rng.normal(0.0, 0.1, ID)))


def activations(rng, T, lda=NA_FULL, outlier_frac=0.01, outlier_scale=20.0, zero_tiles=0):
    """The fp8.a GEMM output [T, lda] bf16 bits: q_a, k_pe, wk ~ N(0, 1); kv_a ~ N(0, 1) with
    `outlier_frac` of its values x `outlier_scale`; `zero_tiles` rows get one all-zero 128-wide kv_a
    tile (amax 0: scale 0)."""
    x = rng.standard_normal((T, lda), dtype=np.float32)
    kv = x[:, QL:QL + KVL]
    mask = rng.random(kv.shape) < outlier_frac
    kv[mask] *= outlier_scale
    if zero_tiles:
        rows = rng.choice(T, size=min(zero_tiles, T), replace=False)
        for r in rows:
            t = int(rng.integers(0, 4))
            kv[r, t * 128:(t + 1) * 128] = 0.0
    return bf16_bits(x)


def rope_table(n_pos):
    """[n_pos, 64] bf16 bits: 32 cos then 32 sin of pos * theta^(-2i/64) (GLM's rope_interleave)."""
    inv = THETA ** (-np.arange(0, ROPE, 2, dtype=np.float64) / ROPE)
    ang = np.arange(n_pos, dtype=np.float64)[:, None] * inv[None, :]
    return bf16_bits(np.concatenate([np.cos(ang), np.sin(ang)], axis=1).astype(np.float32))


def positions(call):
    """pos of every fresh row: its sequence's last fresh[s] positions (glm_glue.cu:118)."""
    return np.concatenate([np.arange(p, p + f, dtype=np.int32) for p, f in zip(call.prefix, call.fresh)])


def topk_indices(rng, call):
    """The indexer's picks [T, 2048] i32, sequence-relative: 2048 distinct positions uniform in
    [0, klen) when klen > 2048, else 0 .. klen - 1 then -1 (vLLM's short-row shortcut)."""
    klen = positions(call).astype(np.int64) + 1
    out = np.full((call.T, TOPK), -1, dtype=np.int32)
    short = np.flatnonzero(klen <= TOPK)
    if len(short):
        ar = np.arange(TOPK)
        out[short] = np.where(ar[None, :] < klen[short, None], ar[None, :], -1)
    mid = np.flatnonzero((klen > TOPK) & (klen <= 4 * TOPK))
    for r in mid:
        out[r] = rng.permutation(int(klen[r]))[:TOPK]
    long_ = np.flatnonzero(klen > 4 * TOPK)
    for lo in range(0, len(long_), 2048):  # in blocks of rows: draw, drop repeats, shuffle, keep 2048
        rows = long_[lo:lo + 2048]
        kl = klen[rows]
        cand = np.sort((rng.random((len(rows), TOPK + TOPK // 2)) * kl[:, None]).astype(np.int64), axis=1)
        rep = np.zeros(cand.shape, dtype=bool)
        rep[:, 1:] = cand[:, 1:] == cand[:, :-1]
        key = np.where(rep, 2.0, rng.random(cand.shape))
        take = np.argsort(key, axis=1)[:, :TOPK]
        picked = np.take_along_axis(cand, take, axis=1)
        ok = (~rep).sum(axis=1) >= TOPK
        out[rows[ok]] = picked[ok]
        for r in rows[~ok]:
            out[r] = rng.permutation(int(klen[r]))[:TOPK]
    return out


def random_latent_pages(rng, n_pages, kv_dtype="fp8"):
    """A latent cache pool of `n_pages` 64-token pages with every byte value in play: e4m3 codes
    uniform over all 256 (NaN codes included unless excluded by the caller), positive f32 tile scales
    spanning 2^-20 .. 2^4, bf16 k_pe ~ N(0, 1). bf16 pools hold N(0, 1) values."""
    if kv_dtype == "bf16":
        return bf16_bits(rng.standard_normal(n_pages * PAGE * 576, dtype=np.float32)).view(np.uint8)
    rows = np.empty((n_pages * PAGE, 656), dtype=np.uint8)
    rows[:, :512] = rng.integers(0, 256, size=(n_pages * PAGE, 512), dtype=np.uint8)
    sc = np.exp2(rng.uniform(-20, 4, size=(n_pages * PAGE, 4))).astype(np.float32)
    rows[:, 512:528] = sc.view(np.uint8)
    rows[:, 528:] = bf16_bits(rng.standard_normal((n_pages * PAGE, 64), dtype=np.float32)).view(np.uint8)
    return rows.reshape(-1)


def random_index_pages(rng, n_pages):
    """An indexer cache pool: e4m3 keys, then per-token UE8M0 power-of-two f32 scales."""
    pages = np.empty((n_pages, PAGE * IDX_ROW), dtype=np.uint8)
    pages[:, :PAGE * ID] = rng.integers(0, 256, size=(n_pages, PAGE * ID), dtype=np.uint8)
    sc = np.exp2(rng.integers(-12, 4, size=(n_pages, PAGE))).astype(np.float32)
    pages[:, PAGE * ID:] = sc.view(np.uint8)
    return pages.reshape(-1)
