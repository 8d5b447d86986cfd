"""Layer groups: GLM-5.3's 78 layers cut into pipeline stages, one stage a GPU.

Every layer owns its latent cache (``kv.<l>``) and, on an indexer layer, its indexer cache
(``idx.<l>``) (kern-glm53 scripts/gen.py:330-332), so layers shard across GPUs with no exchange on
the cache path. A stage starts at an indexer layer, so a shared layer never needs top-k picks from
another stage (gen.py:491); each stage runs its own row plan at its first layer (gen.py:317-329).

``LayerGroup`` holds one stage's states on one device and runs a call's cache path through its
layers in the manifest's order (gen.py:365-398): the append (``mla_prep_full`` / ``_shared``); on an
indexer layer the key gather and the row plan of its top-k picks; the paged dequant.
"""
from dataclasses import dataclass

import torch

from . import ops, traffic

LAYERS = 78
FULL = frozenset({0, 1, 2} | set(range(6, LAYERS, 4)))  # indexer layers (gen.py:59)
PAGE = 64

# The stage cuts of kern-glm53's deployment at 4 GPUs (README.md:13-16, gen.py:484) and the cuts
# this module picks for other counts (balanced by algorithmic bytes, at indexer layers only).
REFERENCE_CUTS = {4: (0, 18, 38, 58)}


def layer_bytes(l, T, ctx, kv_dtype="fp8"):
    return traffic.layer(T, ctx, l in FULL, kv_dtype)


# The slowdown of a stage that sends or receives forwarded picks by copy-engine peer copies
# (dist.PeerCopyForwarder), as measured on B200: 0.3% (7.971 against 7.946 ms a call of 39 layers)
FORWARD_SLOWDOWN = 0.005


def cuts(n_groups, T=16384, ctx=1 << 20, kv_dtype="fp8", any_layer=False):
    """First layers of `n_groups` stages, minimising the largest stage's cost. Each stage starts at an
    indexer layer (the reference's rule, scripts/gen.py:491), or with `any_layer` at any layer: a stage
    that then starts at a shared layer needs the picks of the indexer layer before it from the stage
    that owns that layer (`forwarded_picks`). A stage's cost is its layers' algorithmic bytes; a stage
    that sends or receives picks also pays the forwarded bytes and FORWARD_SLOWDOWN, so the solver cuts
    at a shared layer only where the better balance outweighs the exchange."""
    starts = list(range(LAYERS)) if any_layer else sorted(FULL)
    if n_groups < 1 or n_groups > len(starts):
        raise ValueError(f"{n_groups} stages: between 1 and {len(starts)}")
    w = [layer_bytes(l, T, ctx, kv_dtype) for l in range(LAYERS)]
    pre = [0]
    for x in w:
        pre.append(pre[-1] + x)
    cand = starts + [LAYERS]
    end = len(cand) - 1
    INF = float("inf")
    def stage_cost(a, b):  # layers [a, b): receives picks when a is a shared layer, sends when b is
        c = pre[b] - pre[a]
        recv, send = a not in FULL, b < LAYERS and b not in FULL
        if recv or send:
            c = c * (1 + FORWARD_SLOWDOWN) + picks_bytes(T) * (recv + send)
        return c

    def solve(combine, limit):
        # best[k][i]: the objective for layers [cand[i], 78) in k stages, no stage above `limit`
        best = [[INF] * len(cand) for _ in range(n_groups + 1)]
        nxt = [[None] * len(cand) for _ in range(n_groups + 1)]
        best[0][end] = 0
        for k in range(1, n_groups + 1):
            for i in range(end):
                for j in range(i + 1, len(cand)):
                    c = stage_cost(cand[i], cand[j])
                    if best[k - 1][j] == INF or c > limit:
                        continue
                    v = combine(c, best[k - 1][j])
                    if v < best[k][i]:
                        best[k][i], nxt[k][i] = v, j
        return best, nxt

    # the smallest possible largest stage, then the most even split that keeps to it
    best, _ = solve(max, INF)
    if best[n_groups][0] == INF:
        raise ValueError(f"no split into {n_groups} stages")
    _, nxt = solve(lambda c, rest: c * c + rest, best[n_groups][0])
    out, i = [], 0
    for k in range(n_groups, 0, -1):
        out.append(cand[i])
        i = nxt[k][i]
    return tuple(out)


def picks_bytes(T):
    """Bytes of one forward of a call's picks: ind [T, 2048] i32 and tlen [T] i32."""
    return 4 * T * 2048 + 4 * T


def group_of(rank, n_groups, **kw):
    c = cuts(n_groups, **kw) + (LAYERS,)
    return c[rank], c[rank + 1]


def picks_source(l):
    """The indexer layer whose top-k picks layer `l` attends with: `l` itself on an indexer layer, else
    the last indexer layer before it (a shared layer reuses its picks, scripts/gen.py:388-400)."""
    return max(f for f in FULL if f <= l)


def forwarded_picks(cut_list):
    """[(sender, receiver, source layer)]: for every stage that starts at a shared layer, the stage that
    owns the indexer layer whose picks its first layers use. Empty when every stage starts at an
    indexer layer. Sent per call: the picks [T, 2048] i32 after the row plan, and tlen [T] i32."""
    c = list(cut_list) + [LAYERS]
    owner = lambda l: max(i for i in range(len(c) - 1) if c[i] <= l)
    out = []
    for k in range(1, len(c) - 1):
        if c[k] not in FULL:
            src = picks_source(c[k])
            out.append((owner(src), k, src))
    return out


@dataclass
class CallMeta:
    """A call's metadata on the device (gen.py:212-218): cu_seqlens, seq_lens, block_table, slot_mapping."""
    cu: torch.Tensor
    seq_lens: torch.Tensor
    block_table: torch.Tensor
    slot: torch.Tensor
    nseq: int
    T: int
    ctx: int

    @property
    def max_pages(self):
        return int(self.block_table.shape[1])


@dataclass
class LayerInputs:
    """What the rest of a layer hands the cache path: the fp8.a GEMM output and the norm weights."""
    x: torch.Tensor     # [chunk, 2752] bf16
    g_q: torch.Tensor   # [2048] bf16
    g_kv: torch.Tensor  # [512] bf16
    ik_w: torch.Tensor = None  # [128] bf16, indexer layers
    ik_b: torch.Tensor = None


class LayerGroup:
    """One stage's caches for layers [first, last) on `device`, and its per-call workspaces."""

    def __init__(self, first, last, n_pages, max_ctx, chunk, kv_dtype="fp8", device=None):
        self.first, self.last = first, last
        self.layers = list(range(first, last))
        self.kv_dtype = kv_dtype
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.chunk, self.max_ctx, self.n_pages = chunk, max_ctx, n_pages
        row = 656 if kv_dtype == "fp8" else 1152
        dev = self.device
        self.kv = {l: torch.empty(n_pages * PAGE * row, dtype=torch.uint8, device=dev) for l in self.layers}
        self.idx = {l: torch.empty(n_pages * PAGE * 132, dtype=torch.uint8, device=dev)
                    for l in self.layers if l in FULL}
        i32 = lambda n: torch.empty(n, dtype=torch.int32, device=dev)
        self.pos, self.ks, self.ke, self.klen, self.row_seq, self.zero, self.tlen = (i32(chunk) for _ in range(7))
        self.qq = torch.empty(chunk * 2048, dtype=torch.uint8, device=dev)
        self.sf_rows = chunk
        self.qsf = torch.empty(4 * chunk * 4, dtype=torch.uint8, device=dev)
        self.kg = torch.empty(max_ctx * 128, dtype=torch.uint8, device=dev)
        self.ksf = torch.empty(max_ctx, dtype=torch.float32, device=dev)
        self.kvd = torch.empty(max_ctx * 576, dtype=torch.bfloat16, device=dev) if kv_dtype == "fp8" else None
        self.launches = 0

    def launches_per_call(self):
        n = 1  # the stage's row plan
        for l in self.layers:
            n += 2 if self.kv_dtype == "fp8" else 1
            if l in FULL:
                n += 2
        return n

    def bytes_per_call(self, T, ctx, nseq):
        return traffic.plan(T, nseq) + sum(layer_bytes(l, T, ctx, self.kv_dtype) for l in self.layers)

    def run_call(self, meta: CallMeta, inputs, ind, stream=None, on_dequant=None, on_op=None):
        """The cache path of one call through the group's layers. `inputs[l]` is a LayerInputs,
        `ind[l]` the top-k picks [T, 2048] i32 of indexer layer l (rewritten in place).
        `on_op(op, l, before)` is called around every launch (op one of "plan", "mla_prep",
        "idx_gather", "topk", "kv_dequant"; l None for the stage's plan), and `on_dequant(l, before)`
        around each dequant launch: hooks for per-kernel timing."""
        T, nseq, mp = meta.T, meta.nseq, meta.max_pages
        hook = on_op or (lambda op, l, before: None)
        hook("plan", None, True)
        ops.plan(meta.cu, meta.seq_lens, nseq, self.pos, self.ks, self.ke, self.klen, self.row_seq, self.zero, T,
                 stream=stream)
        hook("plan", None, False)
        for l in self.layers:
            a = inputs[l]
            hook("mla_prep", l, True)
            if l in FULL:
                ops.mla_prep_full(a.x, a.x.shape[1], a.g_q, a.g_kv, self.rope, self.pos, meta.slot, self.kv[l],
                                  self.idx[l], a.ik_w, a.ik_b, self.qq, self.qsf, self.sf_rows, T,
                                  kv_dtype=self.kv_dtype, stream=stream)
                hook("mla_prep", l, False)
                hook("idx_gather", l, True)
                ops.idx_gather(self.idx[l], meta.block_table, mp, meta.seq_lens, nseq, self.kg, self.ksf,
                               stream=stream)
                hook("idx_gather", l, False)
                hook("topk", l, True)
                if self.kv_dtype == "fp8":
                    ops.topk_stream(ind[l], self.ks, self.klen, self.tlen, T, stream=stream)
                else:
                    ops.topk_slots(ind[l], meta.block_table, mp, self.row_seq, self.klen, self.tlen, T, stream=stream)
                hook("topk", l, False)
            else:
                ops.mla_prep_shared(a.x, a.x.shape[1], a.g_q, a.g_kv, self.rope, self.pos, meta.slot, self.kv[l],
                                    self.qq, self.qsf, self.sf_rows, T, kv_dtype=self.kv_dtype, stream=stream)
                hook("mla_prep", l, False)
            if self.kv_dtype == "fp8":
                if on_dequant:
                    on_dequant(l, True)
                hook("kv_dequant", l, True)
                ops.kv_dequant(self.kv[l], meta.block_table, mp, meta.seq_lens, nseq, self.kvd, stream=stream)
                hook("kv_dequant", l, False)
                if on_dequant:
                    on_dequant(l, False)
        self.launches += self.launches_per_call()

    rope = None  # [max_pos, 64] bf16, set by the owner (the rope table is a model constant)
