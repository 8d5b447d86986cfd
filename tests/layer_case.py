"""One layer's cache-path inputs for a seeded call, as NumPy arrays and as device tensors.

Shared by the GPU parity tests, the golden-fixture generator and ``__graft_entry__.smoke``.
"""
import numpy as np

from glmkv import workload as W

QSF_WORDS = W.QL // 512


class LayerCase:
    """Inputs of one layer of `call`: activations, weights, rope, caches with a random prefix, top-k."""

    def __init__(self, call, kv_dtype="fp8", seed=1, zero_tiles=0, nan_codes=True, with_topk=True):
        rng = np.random.default_rng(seed)
        self.call, self.kv_dtype = call, kv_dtype
        self.T = call.T
        self.sf_rows = max(self.T, 1)
        self.w = W.weights(rng)
        self.x = W.activations(rng, self.T, zero_tiles=zero_tiles)
        self.lda = self.x.shape[1]
        self.rope = W.rope_table(int(call.seq_lens.max()))
        self.pos = W.positions(call)
        self.kv_pool = W.random_latent_pages(rng, call.n_pages, kv_dtype)
        if kv_dtype == "fp8" and not nan_codes:
            rows = self.kv_pool.reshape(-1, 656)
            q = rows[:, :512]
            q[(q & 0x7F) == 0x7F] &= 0xFE
        self.idx_pool = W.random_index_pages(rng, call.n_pages)
        self.ind = W.topk_indices(rng, call) if with_topk else None

    # ---------------------------------------------------------------------------------- device side
    def device(self, torch, dev):
        """Fresh device tensors (a dict) for one run of the path."""
        c = self.call
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        d = {
            "x": t(self.x.view(np.int16)).view(torch.bfloat16),
            "g_q": t(self.w.g_q.view(np.int16)).view(torch.bfloat16),
            "g_kv": t(self.w.g_kv.view(np.int16)).view(torch.bfloat16),
            "ik_w": t(self.w.ik_w.view(np.int16)).view(torch.bfloat16),
            "ik_b": t(self.w.ik_b.view(np.int16)).view(torch.bfloat16),
            "rope": t(self.rope.view(np.int16)).view(torch.bfloat16),
            "cu": t(c.cu),
            "seq_lens": t(c.seq_lens),
            "block_table": t(c.block_table),
            "slot": t(c.slot_mapping),
            "kv": t(self.kv_pool),
            "idx": t(self.idx_pool),
            "qq": torch.zeros(max(self.T, 1) * W.QL, dtype=torch.uint8, device=dev),
            "qsf": torch.zeros(QSF_WORDS * self.sf_rows * 4, dtype=torch.uint8, device=dev),
            "kg": torch.zeros(max(c.ctx, 1) * W.ID, dtype=torch.uint8, device=dev),
            "ksf": torch.zeros(max(c.ctx, 1), dtype=torch.float32, device=dev),
            "kvd": torch.zeros(max(c.ctx, 1) * 576, dtype=torch.bfloat16, device=dev),
            "tlen": torch.zeros(max(self.T, 1), dtype=torch.int32, device=dev),
        }
        for k in ("pos", "klen", "row_seq", "zero"):
            d[k] = torch.zeros(max(self.T, 1), dtype=torch.int32, device=dev)
        for k in ("ks", "ke"):
            d[k] = torch.zeros(max(self.T, 1), dtype=torch.int32, device=dev)
        if self.ind is not None:
            d["ind"] = t(self.ind)
        return d

    # ---------------------------------------------------------------------------------- oracle side
    def host(self):
        """Fresh host arrays for one run of the C oracle."""
        c = self.call
        return {
            "cu": c.cu.copy(), "seq_lens": c.seq_lens.copy(), "block_table": c.block_table.copy(),
            "slot": c.slot_mapping.copy(), "x": self.x, "rope": self.rope,
            "kv": self.kv_pool.copy(), "idx": self.idx_pool.copy(),
            "qq": np.zeros(max(self.T, 1) * W.QL, np.uint8),
            "qsf": np.zeros(QSF_WORDS * self.sf_rows * 4, np.uint8),
            "kg": np.zeros(max(c.ctx, 1) * W.ID, np.uint8),
            "ksf": np.zeros(max(c.ctx, 1), np.float32),
            "kvd": np.zeros(max(c.ctx, 1) * 576, np.uint16),
            "tlen": np.zeros(max(self.T, 1), np.int32),
            "pos": np.zeros(max(self.T, 1), np.int32), "klen": np.zeros(max(self.T, 1), np.int32),
            "row_seq": np.zeros(max(self.T, 1), np.int32), "zero": np.ones(max(self.T, 1), np.int32),
            "ks": np.zeros(max(self.T, 1), np.uint32), "ke": np.zeros(max(self.T, 1), np.uint32),
            "ind": None if self.ind is None else self.ind.copy(),
        }


def run_glmkv(case, d, full=True, torch=None):
    """The whole path of one layer through libglmkv, in manifest order (kern-glm53 gen.py:318-398)."""
    import glmkv

    c, T = case.call, case.T
    glmkv.plan(d["cu"], d["seq_lens"], c.nseq, d["pos"], d["ks"], d["ke"], d["klen"], d["row_seq"], d["zero"], T)
    if full:
        glmkv.mla_prep_full(d["x"], case.lda, d["g_q"], d["g_kv"], d["rope"], d["pos"], d["slot"], d["kv"], d["idx"],
                            d["ik_w"], d["ik_b"], d["qq"], d["qsf"], case.sf_rows, T, kv_dtype=case.kv_dtype)
        glmkv.idx_gather(d["idx"], d["block_table"], c.max_pages, d["seq_lens"], c.nseq, d["kg"], d["ksf"])
        if "ind" in d:
            if case.kv_dtype == "fp8":
                glmkv.topk_stream(d["ind"], d["ks"], d["klen"], d["tlen"], T)
            else:
                glmkv.topk_slots(d["ind"], d["block_table"], c.max_pages, d["row_seq"], d["klen"], d["tlen"], T)
    else:
        glmkv.mla_prep_shared(d["x"], case.lda, d["g_q"], d["g_kv"], d["rope"], d["pos"], d["slot"], d["kv"],
                              d["qq"], d["qsf"], case.sf_rows, T, kv_dtype=case.kv_dtype)
    if case.kv_dtype == "fp8":
        glmkv.kv_dequant(d["kv"], d["block_table"], c.max_pages, d["seq_lens"], c.nseq, d["kvd"])


def run_reference(case, d, full=True):
    """The same layer through the reference's own kernels (oracle/_ref), with the manifest grids."""
    from oracle import ref

    c, T = case.call, case.T
    p = lambda k: d[k].data_ptr()
    ref.plan(p("cu"), p("seq_lens"), c.nseq, p("pos"), p("ks"), p("ke"), p("klen"), p("row_seq"), p("zero"), T)
    ref.mla_prep(case.kv_dtype == "fp8", p("x"), case.lda, p("g_q"), p("g_kv"), p("rope"), p("pos"), p("slot"),
                 p("kv"), p("idx") if full else None, p("ik_w") if full else None, p("ik_b") if full else None,
                 p("qq"), p("qsf"), case.sf_rows, T)
    if full:
        ref.idx_gather(p("idx"), p("block_table"), c.max_pages, p("seq_lens"), c.nseq, p("kg"), p("ksf"), c.ctx)
        if "ind" in d:
            if case.kv_dtype == "fp8":
                ref.topk_stream(p("ind"), p("ks"), p("klen"), p("tlen"), T)
            else:
                ref.topk_slots(p("ind"), p("block_table"), c.max_pages, p("row_seq"), p("klen"), p("tlen"), T)
    if case.kv_dtype == "fp8":
        ref.kv_dequant(p("kv"), p("block_table"), c.max_pages, p("seq_lens"), c.nseq, p("kvd"), c.ctx)


def run_oracle(case, h, full=True):
    """The same layer through the C oracle."""
    from oracle import cpu

    c, T = case.call, case.T
    cpu.plan(h["cu"], h["seq_lens"], c.nseq, h["pos"], h["ks"], h["ke"], h["klen"], h["row_seq"], h["zero"], T)
    cpu.mla_prep(case.kv_dtype == "fp8", h["x"], case.lda, case.w.g_q, case.w.g_kv, h["rope"], h["pos"], h["slot"],
                 h["kv"], h["idx"] if full else None, case.w.ik_w if full else None, case.w.ik_b if full else None,
                 h["qq"], h["qsf"], case.sf_rows, T)
    if full:
        cpu.idx_gather(h["idx"], h["block_table"], c.max_pages, h["seq_lens"], c.nseq, h["kg"], h["ksf"])
        if h["ind"] is not None:
            if case.kv_dtype == "fp8":
                cpu.topk_stream(h["ind"], h["ks"], h["klen"], h["tlen"], T)
            else:
                cpu.topk_slots(h["ind"], h["block_table"], c.max_pages, h["row_seq"], h["klen"], h["tlen"], T)
    if case.kv_dtype == "fp8":
        cpu.kv_dequant(h["kv"], h["block_table"], c.max_pages, h["seq_lens"], c.nseq, h["kvd"])


OUTPUTS = ("pos", "ks", "ke", "klen", "row_seq", "zero", "qq", "qsf", "kv", "idx", "kg", "ksf", "kvd", "ind", "tlen")


def to_host(d, torch):
    """Device results as NumPy arrays in the oracle's dtypes."""
    out = {}
    for k in OUTPUTS:
        if k not in d:
            continue
        v = d[k].detach().cpu()
        if v.dtype == torch.bfloat16:
            v = v.view(torch.int16)
        a = v.numpy()
        if k in ("ks", "ke"):
            a = a.view(np.uint32)
        if k == "kvd":
            a = a.view(np.uint16)
        out[k] = a
    return out


LDB = 64 * 256 + 32 * 128  # NB[True] (kern-glm53 scripts/gen.py:63)


def q_post_case(T, seed, ldb=LDB):
    """Inputs of glm_q_post: q_b's output [T, ldb] bf16 (scaled N(0, 1) rows), rope, positions, iw."""
    rng = np.random.default_rng(seed)
    qb = np.zeros((T, ldb), np.uint16)
    qb[:, :LDB] = W.bf16_bits(rng.standard_normal((T, LDB), dtype=np.float32) * rng.uniform(0.1, 8, (T, 1)))
    n_pos = 4096
    return {"qb": qb, "rope": W.rope_table(n_pos), "pos": rng.integers(0, n_pos, T).astype(np.int32),
            "iw": W.bf16_bits(rng.standard_normal((T, 32), dtype=np.float32)), "T": T, "ldb": ldb}




def norm_case(T, seed, with_a=True):
    """Inputs of glm_add_rms_quant: a, res [T, 6144] bf16 (rows scaled 0.05 .. 20; row 1 all zero), gamma."""
    H = 6144
    rng = np.random.default_rng(seed)
    scale = rng.uniform(0.05, 20, (T, 1)).astype(np.float32)
    res = W.bf16_bits(rng.standard_normal((T, H), dtype=np.float32) * scale)
    a = W.bf16_bits(rng.standard_normal((T, H), dtype=np.float32) * scale) if with_a else None
    gamma = W.bf16_bits(rng.uniform(0.5, 1.5, H).astype(np.float32))
    if T > 2:
        res[1] = 0  # an all-zero row (a too): rr = rsqrt(eps)
        if a is not None:
            a[1] = 0
    return a, res, gamma


def quant_case(T, K, ldx):
    """Input of glm_quant: x [T, ldx] bf16, rows scaled 1e-3 .. 1e3, one all-zero block."""
    rng = np.random.default_rng(T + K)
    x = W.bf16_bits(rng.standard_normal((T, ldx), dtype=np.float32) * rng.uniform(1e-3, 1e3, (T, 1)))
    if T > 2:
        x[1, :128] = 0  # an all-zero block: scale from eps 1e-10
    return x
