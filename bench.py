#!/usr/bin/env python3
"""Benchmark of GLM-5.3's prefill KV-cache path on B200: fp8 KV append + paged dequant GB/s (% of HBM
peak), tokens/s, at 1/2/4/8 GPUs by layer groups.

A step is one packed prefill call (cfg3: 16 sequences, 16,384 fresh rows, prefixes from {0, 2K, 64K,
256K}, at most 2^20 stream tokens) through the cache path of all 78 layers: per stage its row plan,
then per layer the append (fp8 latent row + q quant, and the indexer key on indexer layers), on
indexer layers the key gather and the top-k row plan, and the paged dequant of every sequence's
prefix + chunk. With N GPUs the 78 layers are cut into N stages, one stage a GPU (pipeline
parallelism, as the reference deploys it): at indexer layers, or also at shared layers where that
balances better, with the picks of the indexer layer before such a cut copied to the next stage once a
call (copy-engine peer copies; the one transfer on the data path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl glmkv|reference] [--workload cfg3|cfg1|cfg2]
    torchrun --nproc-per-node N bench.py --gpus N ...

Rank 0 prints one JSON line. `value` is the whole job's algorithmic bytes over the slowest rank's
device time (inputs resident in HBM); `e2e` repeats the measurement through the public API with the
call's metadata copied in from pinned host memory and the row-plan lengths read back every step.
`--impl reference` runs the same workload through the reference's own glue kernels (kern-glm53
source/glm_glue.cu compiled from source, oracle/_ref) with the manifest's launch grids.
"""
import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT), str(ROOT / "kern-glm53_b200")]

METRIC = "fp8 KV append+paged dequant GB/s (% HBM peak), tokens/s at 1/2/4/8 B200"
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0  # the pool's earlier burst measurement, used when MEASURED_PEAKS.json is absent
WORKLOADS = {
    "cfg3": "cfg3: one 16-sequence / 16,384-row prefill call through the cache path of all 78 layers, "
            "prefixes from {0, 2K, 64K, 256K}, stream <= 2^20 tokens, fp8 latent cache + indexer cache",
    "cfg1": "cfg1: one 16-sequence / 16,384-row call (prefixes U[0, 32768]) through one indexer layer",
    "cfg2": "cfg2: one 2^20-token sequence (16,384 fresh rows) through one indexer layer",
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("glmkv", "reference"), default="glmkv")
    ap.add_argument("--workload", choices=tuple(WORKLOADS), default="cfg3")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cfg2", action="store_true", help="skip the 1M-context (cfg2) layer block")
    ap.add_argument("--no-marked", action="store_true", help="skip the row-selective lift block")
    ap.add_argument("--cuts", default=None, help="first layers of the stages, comma-separated (overrides --placement)")
    ap.add_argument("--placement", choices=("any", "indexer"), default="any",
                    help="stage cuts at any layer, with the picks forwarded to a stage that starts at a shared "
                         "layer (default), or at indexer layers only (the reference's deployment rule)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--no-next-rows", action="store_true",
                    help="skip timing the ops beside the path (q_post, add_rms_quant, quant, MQA logits) "
                         "and the bf16-cache path")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU-baseline sample budget")
    return ap.parse_args()


def measured_peak(key="hbm_gbs"):
    """The pool's measured peak (`hbm_gbs` GB/s, or `bf16_tflops` TFLOP/s) and whether it was measured."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())[key]), "measured"
        except (KeyError, ValueError):
            pass
    return (FALLBACK_HBM_GBS if key == "hbm_gbs" else FALLBACK_BF16_TFLOPS), "fallback"


# ------------------------------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi clocks / throttle reasons of the given GPUs, sampled while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, ids, enabled=True):
        self.ids, self.proc, self.lines = ids, None, []
        self.enabled = enabled

    def __enter__(self):
        if self.enabled:
            try:
                cmd = ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "50"]
                if self.ids:
                    cmd += ["-i", ",".join(self.ids)]
                self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                # the sampler is running before the timed region starts (at 8 GPUs that region can be
                # shorter than nvidia-smi's start-up): wait for its first sample, at most 5 s
                import select
                if select.select([self.proc.stdout], [], [], 5.0)[0]:
                    first = self.proc.stdout.readline()
                    if first.strip():
                        self.lines.append(first.strip())
            except OSError:
                self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines += [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons, pw = [], [], set(), []
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
                pw.append(float(f[3]))
            except ValueError:
                continue
            for name, v in zip(self.REASONS, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(pw)}


# ------------------------------------------------------------------------------------------ setup

def device_call(torch, call, dev):
    from glmkv.stage import CallMeta

    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return CallMeta(t(call.cu), t(call.seq_lens), t(call.block_table), t(call.slot_mapping), call.nseq, call.T,
                    call.ctx)


def fill_caches(torch, group, gen):
    """Prefix caches of every layer: random e4m3 codes (NaN codes excluded), positive f32 tile scales,
    N(0, 1) bf16 k_pe; indexer pages with power-of-two scales."""
    for l, kv in group.kv.items():
        kv.copy_(torch.randint(0, 256, kv.shape, dtype=torch.uint8, device=kv.device, generator=gen))
        nan = (kv & 0x7F) == 0x7F
        kv.sub_(nan.to(torch.uint8))
        del nan
        rows = kv.view(-1, 656)
        sc = torch.exp2(torch.rand(rows.shape[0], 4, device=kv.device, generator=gen) * 12 - 10)
        rows[:, 512:528] = sc.view(torch.uint8).view(-1, 16)
        pe = torch.randn(rows.shape[0], 64, device=kv.device, generator=gen).to(torch.bfloat16)
        rows[:, 528:] = pe.view(torch.uint8).view(-1, 128)
    for l, idx in group.idx.items():
        idx.copy_(torch.randint(0, 256, idx.shape, dtype=torch.uint8, device=idx.device, generator=gen))
        pages = idx.view(-1, 64 * 132)
        sc = torch.exp2(torch.randint(-12, 4, (pages.shape[0], 64), device=idx.device, generator=gen).float())
        pages[:, 8192:] = sc.view(torch.uint8).view(-1, 256)


def layer_inputs(torch, group, T, gen):
    """Per layer: the fp8.a GEMM output [T, 2752] (N(0,1); kv_a with 1% x20 outliers) and the norm weights."""
    from glmkv.stage import FULL, LayerInputs

    dev = group.device
    out = {}
    for l in group.layers:
        x = torch.randn(T, 2752, device=dev, generator=gen)
        kv = x[:, 2048:2560]
        kv.mul_(torch.where(torch.rand(kv.shape, device=dev, generator=gen) < 0.01, 20.0, 1.0))
        u = lambda n: (torch.rand(n, device=dev, generator=gen) + 0.5).to(torch.bfloat16)
        out[l] = LayerInputs(x.to(torch.bfloat16), u(2048), u(512), u(128) if l in FULL else None,
                             (torch.randn(128, device=dev, generator=gen) * 0.1).to(torch.bfloat16) if l in FULL else None)
        del x
    return out


def topk_picks(torch, call, group, gen, layers=None):
    """Per indexer layer (of `layers`, default the group's): 2048 positions uniform in [0, klen) per row
    (drawn with replacement on the device), or 0 .. klen - 1 then -1 when klen <= 2048."""
    from glmkv import workload as W
    from glmkv.stage import FULL

    dev = group.device
    klen = torch.from_numpy(W.positions(call).astype(np.int64) + 1).to(dev)
    ar = torch.arange(2048, device=dev)
    short = (ar[None, :] < klen[:, None]).to(torch.int32) * (ar[None, :].to(torch.int32) + 1) - 1
    out = {}
    for l in (group.layers if layers is None else layers):
        if l not in FULL:
            continue
        pick = (torch.rand(call.T, 2048, device=dev, generator=gen) * klen[:, None]).to(torch.int32)
        out[l] = torch.where((klen <= 2048)[:, None], short, pick).contiguous()
    return out


# ------------------------------------------------------------------------------------------ the reference arm

def run_call_reference(group, meta, inputs, ind, ctx, on_dequant=None, on_op=None):
    """The same call through the reference's own kernels (oracle/_ref), manifest launch grids. The hooks
    are LayerGroup.run_call's."""
    from glmkv.stage import FULL
    from oracle import ref

    p = lambda t: t.data_ptr()
    hook = on_op or (lambda op, l, before: None)
    T, nseq, mp = meta.T, meta.nseq, meta.max_pages
    hook("plan", None, True)
    ref.plan(p(meta.cu), p(meta.seq_lens), nseq, p(group.pos), p(group.ks), p(group.ke), p(group.klen),
             p(group.row_seq), p(group.zero), T)
    hook("plan", None, False)
    for l in group.layers:
        a = inputs[l]
        full = l in FULL
        hook("mla_prep", l, True)
        ref.mla_prep(True, p(a.x), a.x.shape[1], p(a.g_q), p(a.g_kv), p(group.rope), p(group.pos), p(meta.slot),
                     p(group.kv[l]), p(group.idx[l]) if full else None, p(a.ik_w) if full else None,
                     p(a.ik_b) if full else None, p(group.qq), p(group.qsf), group.sf_rows, T)
        hook("mla_prep", l, False)
        if full:
            hook("idx_gather", l, True)
            ref.idx_gather(p(group.idx[l]), p(meta.block_table), mp, p(meta.seq_lens), nseq, p(group.kg),
                           p(group.ksf), ctx)
            hook("idx_gather", l, False)
            hook("topk", l, True)
            ref.topk_stream(p(ind[l]), p(group.ks), p(group.klen), p(group.tlen), T)
            hook("topk", l, False)
        if on_dequant:
            on_dequant(l, True)
        hook("kv_dequant", l, True)
        ref.kv_dequant(p(group.kv[l]), p(meta.block_table), mp, p(meta.seq_lens), nseq, p(group.kvd), ctx)
        hook("kv_dequant", l, False)
        if on_dequant:
            on_dequant(l, False)


def compose(*hooks):
    """One on_op hook that calls each of `hooks` (None entries skipped) in order."""
    hs = [h for h in hooks if h is not None]
    if not hs:
        return None
    if len(hs) == 1:
        return hs[0]
    return lambda op, l, before: [h(op, l, before) for h in hs] and None


class OpTimer:
    """CUDA events on the launch stream around every kernel of one target layer a step (and around the
    stage's row plan every step): per-kernel device time inside the timed region."""
    KERNELS = {"plan": "glm_plan", "mla_prep.indexer_layer": "glm_mla_prep_fp8",
               "mla_prep.shared_layer": "glm_mla_prep_fp8", "idx_gather": "glm_idx_gather",
               "topk": "glm_topk_stream", "kv_dequant": "glm_kv_dequant"}

    def __init__(self, torch):
        self.torch, self.target, self.open, self.spans = torch, None, {}, {}

    @staticmethod
    def key(op, l):
        from glmkv.stage import FULL
        if op == "mla_prep":
            return "mla_prep.indexer_layer" if l in FULL else "mla_prep.shared_layer"
        return op

    def __call__(self, op, l, before):
        if op != "plan" and l != self.target:
            return
        e = self.torch.cuda.Event(enable_timing=True)
        e.record()
        k = self.key(op, l)
        if before:
            self.open[k] = e
        else:
            self.spans.setdefault(k, []).append((self.open.pop(k), e))

    def mean_us(self, k):
        sp = self.spans.get(k, [])
        return sum(a.elapsed_time(b) for a, b in sp) / len(sp) * 1e3 if sp else None

    def per_op(self, call, peak):
        """{op: kernel, launches timed, mean us, algorithmic bytes a launch, GB/s, fraction of `peak`}."""
        from glmkv import traffic

        nbytes = {"plan": traffic.plan(call.T, call.nseq), "mla_prep.indexer_layer": traffic.mla_prep(call.T, True),
                  "mla_prep.shared_layer": traffic.mla_prep(call.T, False), "idx_gather": traffic.idx_gather(call.ctx),
                  "topk": traffic.topk(call.T), "kv_dequant": traffic.kv_dequant(call.ctx)}
        out = {}
        for k, b in nbytes.items():
            us = self.mean_us(k)
            if us is None:
                continue
            gbs = b / us / 1e3
            out[k] = {"kernel": self.KERNELS[k], "launches_timed": len(self.spans[k]), "us": round(us, 2),
                      "algorithmic_bytes": b, "GB/s": round(gbs, 1), "frac": round(gbs / peak, 4)}
        us = self.mean_us("mla_prep.shared_layer")
        if us is not None:
            b = 1808 * call.T
            out["kv_append_slice"] = {
                "bytes_per_fresh_row": 1808, "algorithmic_bytes": b, "us": round(us, 2),
                "GB/s": round(b / us / 1e3, 1), "frac": round(b / us / 1e3 / peak, 4),
                "note": "the latent-row slice of the append alone (kv_a + k_pe read, the 656-byte fp8 row "
                        "written) over the whole append kernel's time on a shared layer, which also quantizes q"}
        return out


# ------------------------------------------------------------------------------------------ next rows

def next_rows(torch, impl, T, dev, reps=10):
    """The rows beside the path (glm_q_post on an indexer and a shared layer of the same call),
    timed with CUDA events: the mean of `reps` launches after two warm-up launches."""
    from glmkv import traffic
    from glmkv import workload as W

    import glmkv
    g = torch.Generator(device=dev).manual_seed(5)
    ldb = 64 * 256 + 32 * 128
    qb = torch.randn(T, ldb, device=dev, generator=g).to(torch.bfloat16)
    rope = torch.from_numpy(W.rope_table(1 << 16).view(np.int16)).to(dev).view(torch.bfloat16)
    pos = torch.randint(0, 1 << 16, (T,), device=dev, generator=g, dtype=torch.int32)
    qmla = torch.empty(T * 64 * 576, dtype=torch.bfloat16, device=dev)
    iq = torch.empty(T * 32 * 128, dtype=torch.uint8, device=dev)
    iw = torch.randn(T * 32, device=dev, generator=g).to(torch.bfloat16)
    wout = torch.empty(T * 32, dtype=torch.float32, device=dev)
    out = {}
    for full in (True, False):
        if impl == "glmkv":
            if full:
                fn = lambda: glmkv.q_post_full(qb, ldb, rope, pos, qmla, iq, iw, wout, 1, T)
            else:
                fn = lambda: glmkv.q_post_shared(qb, ldb, rope, pos, qmla, 0, T)
        else:
            from oracle import ref
            p = lambda t: t.data_ptr()
            fn = lambda: ref.q_post(p(qb), ldb, p(rope), p(pos), p(qmla), p(iq) if full else None,
                                    p(iw) if full else None, p(wout) if full else None, int(full), T)
        for _ in range(2):
            fn()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        for _ in range(reps):
            fn()
        e.record()
        torch.cuda.synchronize()
        us = s.elapsed_time(e) / reps * 1e3
        nbytes = traffic.q_post(T, full)
        out["indexer_layer" if full else "shared_layer"] = {"us": round(us, 2), "GB/s": round(nbytes / us / 1e3, 1),
                                                            "algorithmic_bytes": nbytes}
    rows = {"glm_q_post": {"rows": T, **out}}
    del qb, qmla, iq, iw, wout
    # the norm + quant glue of a layer: norm_in / norm_post (add_rms_quant) and quant_o (glm_quant)
    H, K = 6144, 64 * 256
    a_ = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
    res_ = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
    gam = (torch.rand(H, device=dev, generator=g) + 0.5).to(torch.bfloat16)
    nrm = torch.empty_like(res_)
    qh = torch.empty(T * H, dtype=torch.uint8, device=dev)
    sfh = torch.empty(H // 512 * T * 4, dtype=torch.uint8, device=dev)
    xo = torch.randn(T, K, device=dev, generator=g).to(torch.bfloat16)
    qo = torch.empty(T * K, dtype=torch.uint8, device=dev)
    sfo = torch.empty(K // 512 * T * 4, dtype=torch.uint8, device=dev)
    if impl == "glmkv":
        f_arq = lambda: glmkv.add_rms_quant(a_, res_, gam, nrm, qh, sfh, T, T)
        f_q = lambda: glmkv.quant_o(xo, K, qo, sfo, T, K, T)
    else:
        from oracle import ref
        p = lambda t: t.data_ptr()
        f_arq = lambda: ref.add_rms_quant(p(a_), p(res_), p(gam), p(nrm), p(qh), p(sfh), T, T)
        f_q = lambda: ref.quant(p(xo), K, p(qo), p(sfo), T, K, T)
    for name, fn, nbytes in (("glm_add_rms_quant", f_arq, traffic.add_rms_quant(T)),
                             ("glm_quant", f_q, traffic.quant(T, K))):
        for _ in range(2):
            fn()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        for _ in range(reps):
            fn()
        e.record()
        torch.cuda.synchronize()
        us = s.elapsed_time(e) / reps * 1e3
        rows[name] = {"rows": T, "us": round(us, 2), "GB/s": round(nbytes / us / 1e3, 1), "algorithmic_bytes": nbytes}
    rows["glm_quant"]["K"] = K
    return rows


def bf16_rows(torch, impl, group, meta, call, dev, reps=10):
    """The bf16-cache path of the manifest (`--kv bf16`, gen.py:53): the append into a bf16 latent cache
    (glm_mla_prep) on an indexer and a shared layer of the call, and the picks mapped to cache slots
    through the page table (glm_topk_slots). glm_topk_slots rewrites its picks in place, so each of its
    launches gets fresh picks copied in before its own events; the appends are timed as a run of
    `reps` launches."""
    from glmkv import traffic
    from glmkv.stage import FULL

    layers = [l for l in group.layers if l in FULL]
    if not layers:
        return {"unavailable": "no indexer layer in this stage"}
    import glmkv
    T = call.T
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(T, 2752, device=dev, generator=g).to(torch.bfloat16)
    u = lambda n: (torch.rand(n, device=dev, generator=g) + 0.5).to(torch.bfloat16)
    g_q, g_kv, ik_w = u(2048), u(512), u(128)
    ik_b = (torch.randn(128, device=dev, generator=g) * 0.1).to(torch.bfloat16)
    kvb = torch.empty(call.n_pages * 64 * 1152, dtype=torch.uint8, device=dev)
    idx = group.idx[layers[0]]
    picks = topk_picks(torch, call, group, g, layers[:1])[layers[0]]
    ind = torch.empty_like(picks)
    p = lambda t: t.data_ptr()
    if impl == "glmkv":
        def prep(full):
            if full:
                glmkv.mla_prep_full(x, 2752, g_q, g_kv, group.rope, group.pos, meta.slot, kvb, idx, ik_w, ik_b,
                                    group.qq, group.qsf, group.sf_rows, T, kv_dtype="bf16")
            else:
                glmkv.mla_prep_shared(x, 2752, g_q, g_kv, group.rope, group.pos, meta.slot, kvb, group.qq,
                                      group.qsf, group.sf_rows, T, kv_dtype="bf16")
        slots = lambda: glmkv.topk_slots(ind, meta.block_table, call.max_pages, group.row_seq, group.klen,
                                         group.tlen, T)
    else:
        from oracle import ref

        def prep(full):
            ref.mla_prep(False, p(x), 2752, p(g_q), p(g_kv), p(group.rope), p(group.pos), p(meta.slot), p(kvb),
                         p(idx) if full else None, p(ik_w) if full else None, p(ik_b) if full else None,
                         p(group.qq), p(group.qsf), group.sf_rows, T)
        slots = lambda: ref.topk_slots(p(ind), p(meta.block_table), call.max_pages, p(group.row_seq),
                                       p(group.klen), p(group.tlen), T)
    out = {}
    for full in (True, False):
        for _ in range(2):
            prep(full)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        for _ in range(reps):
            prep(full)
        e.record()
        torch.cuda.synchronize()
        us = s.elapsed_time(e) / reps * 1e3
        nbytes = traffic.mla_prep(T, full, "bf16")
        out["indexer_layer" if full else "shared_layer"] = {"us": round(us, 2), "GB/s": round(nbytes / us / 1e3, 1),
                                                            "algorithmic_bytes": nbytes}
    total = 0.0
    for i in range(reps + 2):
        ind.copy_(picks)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        slots()
        e.record()
        torch.cuda.synchronize()
        if i >= 2:
            total += s.elapsed_time(e) * 1e3
    us = total / reps
    nbytes = traffic.topk(T)
    del x, kvb, picks, ind
    return {"glm_mla_prep": {"rows": T, "kv_cache": "bf16 (1152 B/token)", **out},
            "glm_topk_slots": {"rows": T, "us": round(us, 2), "GB/s": round(nbytes / us / 1e3, 1),
                               "algorithmic_bytes": nbytes}}


def mqa_row(torch, impl, group, meta, call, dev, reps=3, sub=1024):
    """The indexer's MQA logits of the call's rows over their sequences' keys, read from the first
    indexer layer's cache pages (glm_mqa_logits_paged), in sub-chunks of `sub` rows as the manifest runs
    the indexer (scripts/gen.py:483, --sub 1024): FLOPs = 2 x 32 heads x 128 dims x sum of klen."""
    from glmkv import workload as W
    from glmkv.stage import FULL

    if impl != "glmkv":
        return {"unavailable": "the reference's MQA logits kernel is DeepGEMM's, an empty submodule in kern-glm53"}
    layers = [l for l in group.layers if l in FULL]
    if not layers:
        return {"unavailable": "no indexer layer in this stage"}
    import glmkv
    T = call.T
    klen = W.positions(call).astype(np.int64) + 1
    stride = int(klen.max())
    g = torch.Generator(device=dev).manual_seed(6)
    iq = torch.randint(0, 126, (T * 32 * 128,), dtype=torch.uint8, device=dev, generator=g)
    w = torch.randn(T, 32, device=dev, generator=g)
    logits = torch.empty(sub * stride, dtype=torch.float32, device=dev)
    idx = group.idx[layers[0]]

    def fn():
        for j in range(0, T, sub):
            glmkv.mqa_logits_paged(iq[j * 4096:], idx, call.n_pages, meta.block_table, call.max_pages,
                                   group.row_seq[j:], group.klen[j:], w[j:], logits, stride, min(sub, T - j))
    fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        fn()
    e.record()
    torch.cuda.synchronize()
    us = s.elapsed_time(e) / reps * 1e3
    flops = int(klen.sum()) * 32 * 128 * 2
    peak, kind = measured_peak("bf16_tflops")
    fp8_peak = 2 * peak
    tf = flops / us / 1e6
    del iq, w, logits
    return {"rows": T, "sub_rows": sub, "keys_scored": int(klen.sum()), "us": round(us, 1), "TFLOP/s": round(tf, 1),
            "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": round(fp8_peak, 1), "unit": "TFLOP/s",
                         "frac": round(tf / fp8_peak, 4),
                         "peak_note": f"dense e4m3 = 2 x the {kind} bf16 GEMM rate (MEASURED_PEAKS.json bf16_tflops)"}}


def isolated_ops(torch, impl, group, meta, inputs, ind, call, peak, passes=2):
    """Each kernel of the path launched back to back over the stage's layers (each launch on its own
    layer's inputs and cache state, all larger than L2), `passes` times, after one untimed pass: the
    kernel's own rate, with the write-back of the launch before it being the same kernel's. Events
    bracket each run of launches."""
    from glmkv import ops, traffic
    from glmkv.stage import FULL

    T, nseq, mp = call.T, call.nseq, meta.max_pages
    full = [l for l in group.layers if l in FULL]
    shared = [l for l in group.layers if l not in FULL]
    pp = lambda t: t.data_ptr()
    if impl == "glmkv":
        def prep(l):
            a = inputs[l]
            if l in FULL:
                ops.mla_prep_full(a.x, a.x.shape[1], a.g_q, a.g_kv, group.rope, group.pos, meta.slot, group.kv[l],
                                  group.idx[l], a.ik_w, a.ik_b, group.qq, group.qsf, group.sf_rows, T)
            else:
                ops.mla_prep_shared(a.x, a.x.shape[1], a.g_q, a.g_kv, group.rope, group.pos, meta.slot, group.kv[l],
                                    group.qq, group.qsf, group.sf_rows, T)
        gather = lambda l: ops.idx_gather(group.idx[l], meta.block_table, mp, meta.seq_lens, nseq, group.kg, group.ksf)
        topk = lambda l: ops.topk_stream(ind[l], group.ks, group.klen, group.tlen, T)
        dequant = lambda l: ops.kv_dequant(group.kv[l], meta.block_table, mp, meta.seq_lens, nseq, group.kvd)
    else:
        from oracle import ref

        def prep(l):
            a = inputs[l]
            f = l in FULL
            ref.mla_prep(True, pp(a.x), a.x.shape[1], pp(a.g_q), pp(a.g_kv), pp(group.rope), pp(group.pos),
                         pp(meta.slot), pp(group.kv[l]), pp(group.idx[l]) if f else None, pp(a.ik_w) if f else None,
                         pp(a.ik_b) if f else None, pp(group.qq), pp(group.qsf), group.sf_rows, T)
        gather = lambda l: ref.idx_gather(pp(group.idx[l]), pp(meta.block_table), mp, pp(meta.seq_lens), nseq,
                                          pp(group.kg), pp(group.ksf), call.ctx)
        topk = lambda l: ref.topk_stream(pp(ind[l]), pp(group.ks), pp(group.klen), pp(group.tlen), T)
        dequant = lambda l: ref.kv_dequant(pp(group.kv[l]), pp(meta.block_table), mp, pp(meta.seq_lens), nseq,
                                           pp(group.kvd), call.ctx)
    runs = [("mla_prep.indexer_layer", "glm_mla_prep_fp8", prep, full, traffic.mla_prep(T, True)),
            ("mla_prep.shared_layer", "glm_mla_prep_fp8", prep, shared, traffic.mla_prep(T, False)),
            ("idx_gather", "glm_idx_gather", gather, full, traffic.idx_gather(call.ctx)),
            ("topk", "glm_topk_stream", topk, full, traffic.topk(T)),
            ("kv_dequant", "glm_kv_dequant", dequant, group.layers, traffic.kv_dequant(call.ctx))]
    out = {}
    for name, kernel, fn, layers, nbytes in runs:
        if not layers:
            continue
        for l in layers:
            fn(l)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        for _ in range(passes):
            for l in layers:
                fn(l)
        e.record()
        torch.cuda.synchronize()
        n = passes * len(layers)
        us = s.elapsed_time(e) / n * 1e3
        gbs = nbytes / us / 1e3
        out[name] = {"kernel": kernel, "launches": n, "us": round(us, 2), "algorithmic_bytes": nbytes,
                     "GB/s": round(gbs, 1), "frac": round(gbs / peak, 4)}
    if "mla_prep.shared_layer" in out:
        us = out["mla_prep.shared_layer"]["us"]
        b = 1808 * T
        out["kv_append_slice"] = {"bytes_per_fresh_row": 1808, "algorithmic_bytes": b, "us": us,
                                  "GB/s": round(b / us / 1e3, 1), "frac": round(b / us / 1e3 / peak, 4)}
    return out


def marked_block(torch, impl, group, meta, call, dev, peak, passes=2):
    """The row-selective lift (glm_mark_rows + glm_kv_dequant_marked) on the call's layers, for two
    pick distributions: the benchmark's uniform picks, and each row's 2048 latest positions (a sliding
    window). The mask is built once from an indexer layer's picks (after the row plan) and serves the
    lift of every layer; the lift is timed back to back over the stage's layers like `isolated_ops`."""
    import glmkv
    from glmkv import traffic
    from glmkv.stage import FULL

    if impl != "glmkv":
        return {"unavailable": "the reference lifts every row: it has no row-selective lift"}
    full = [l for l in group.layers if l in FULL]
    if not full:
        return {"unavailable": "no indexer layer in this stage"}
    T, ctx, mp = call.T, call.ctx, meta.max_pages
    words = (ctx + 63) // 64
    g = torch.Generator(device=dev).manual_seed(11)
    klen = group.klen[:T].to(torch.int64)
    ar = torch.arange(2048, device=dev)
    dists = {"uniform": topk_picks(torch, call, group, g, full[:1])[full[0]],
             "sliding_window": torch.where(ar[None, :] < klen[:, None], (klen[:, None] - 2048).clamp(min=0) + ar[None, :],
                                           -1).to(torch.int32).contiguous()}
    mask = torch.empty(words, dtype=torch.int64, device=dev)
    s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn, n):
        fn()
        torch.cuda.synchronize()
        s_.record()
        for _ in range(n):
            fn()
        e_.record()
        torch.cuda.synchronize()
        return s_.elapsed_time(e_) / n * 1e3

    out = {"note": "mask from one indexer layer's picks after the row plan; lift timed back to back over the "
                   "stage's layers; the full lift (glm_kv_dequant) timed the same way beside it; row_plan_us and "
                   "row_plan_and_mark_fused_us: glm_topk_stream alone and glm_topk_stream_mark, each launch on a "
                   "fresh copy of the sequence-relative picks"}
    lift_all = lambda: [glmkv.kv_dequant(group.kv[l], meta.block_table, mp, meta.seq_lens, call.nseq, group.kvd)
                        for l in group.layers]
    full_us = timed(lift_all, passes) / len(group.layers)
    fresh = torch.empty_like(dists["uniform"])
    tl = torch.empty_like(group.tlen)
    m2 = torch.empty_like(mask)
    s1, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed_fresh(fn, picks, n=6):
        """fn rewrites its picks in place: each launch gets a fresh copy of `picks` before its own events."""
        spans = []
        for i in range(n + 1):
            fresh.copy_(picks)
            s1.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            if i:
                spans.append(s1.elapsed_time(e1) * 1e3)
        return sum(spans) / len(spans)

    for name, picks in dists.items():
        plan_us = timed_fresh(lambda: glmkv.topk_stream(fresh, group.ks, group.klen, tl, T), picks)
        fused_us = timed_fresh(lambda: glmkv.topk_stream_mark(fresh, group.ks, group.klen, tl, T, group.ke, m2, words),
                               picks)
        ind = picks.clone()
        glmkv.topk_stream(ind, group.ks, group.klen, group.tlen, T)
        mark = lambda: glmkv.mark_rows(ind, group.ks, group.ke, T, mask, words)
        mark_us = timed(mark, 5)
        mark()
        lift = lambda: [glmkv.kv_dequant_marked(group.kv[l], meta.block_table, mp, meta.seq_lens, call.nseq, mask,
                                                group.kvd) for l in group.layers]
        lift_us = timed(lift, passes) / len(group.layers)
        bits = np.unpackbits(mask.cpu().numpy().view(np.uint8), bitorder="little")[:ctx].astype(bool)
        # rows read: per page, the span from its first to its last marked row (the whole page when 48
        # or more of its rows are marked); rows written: the marked ones, and all rows of such a page
        goff = np.concatenate([[0], np.cumsum(call.seq_lens)[:-1]])
        read_rows = written = 0
        for s0, ln in zip(goff, call.seq_lens):
            for j in range(0, int(ln), 64):
                page = bits[s0 + j:s0 + min(j + 64, ln)]
                idx = np.flatnonzero(page)
                if idx.size >= 48:
                    read_rows += page.size
                    written += page.size
                elif idx.size:
                    read_rows += int(idx[-1] - idx[0] + 1)
                    written += idx.size
        marked = int(bits.sum())
        lift_bytes = 656 * read_rows + 1152 * written
        mark_bytes = 8192 * T + 8 * words
        out[name] = {"marked_fraction": round(marked / ctx, 4), "rows_marked": marked, "rows_read": read_rows,
                     "rows_written": written,
                     "mark_us": round(mark_us, 2), "mark_GB/s": round(mark_bytes / mark_us / 1e3, 1),
                     "lift_us": round(lift_us, 2), "lift_algorithmic_bytes": lift_bytes,
                     "lift_GB/s": round(lift_bytes / lift_us / 1e3, 1),
                     "lift_frac": round(lift_bytes / lift_us / 1e3 / peak, 4),
                     "full_lift_us": round(full_us, 2),
                     "full_lift_bytes": traffic.kv_dequant(ctx),
                     "speedup_vs_full_lift_incl_mark_every_4_layers": round(full_us / (lift_us + mark_us / 4), 3),
                     # the row plan and the mark in one pass (glm_topk_stream_mark) against the row plan
                     # alone: what marking adds when fused
                     "row_plan_us": round(plan_us, 2), "row_plan_and_mark_fused_us": round(fused_us, 2),
                     "speedup_vs_full_lift_incl_fused_mark_every_4_layers":
                         round(full_us / (lift_us + max(fused_us - plan_us, 0.0) / 4), 3)}
        del ind
    return out


# ------------------------------------------------------------------------------------------ the 1M-context call

def cfg2_block(torch, impl, dev, seed, peak, steps=20, warmup=3):
    """cfg2 (one sequence of 2^20 stream tokens, 16,384 fresh rows) through one indexer layer: the
    whole layer's GB/s over `steps` timed steps, then each kernel's time in `steps` more steps with
    events around every launch."""
    from glmkv import stage, traffic, workload as W

    call = W.config("cfg2", seed=seed)
    group = stage.LayerGroup(0, 1, n_pages=call.n_pages, max_ctx=call.ctx, chunk=call.T, device=dev)
    gen = torch.Generator(device=dev).manual_seed(777 + seed)
    group.rope = torch.from_numpy(W.rope_table(int(call.seq_lens.max())).view(np.int16)).to(dev).view(torch.bfloat16)
    fill_caches(torch, group, gen)
    inputs = layer_inputs(torch, group, call.T, gen)
    ind = topk_picks(torch, call, group, gen)
    meta = device_call(torch, call, dev)
    if impl == "glmkv":
        run = lambda hook=None: group.run_call(meta, inputs, ind, on_op=hook)
    else:
        run = lambda hook=None: run_call_reference(group, meta, inputs, ind, call.ctx, on_op=hook)
    for _ in range(warmup):
        run()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for _ in range(steps):
        run()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / steps
    timer = OpTimer(torch)
    timer.target = 0
    for _ in range(steps):
        run(timer)
    torch.cuda.synchronize()
    nbytes = traffic.plan(call.T, call.nseq) + stage.layer_bytes(0, call.T, call.ctx)
    out = {"workload": WORKLOADS["cfg2"], "seed": seed, "stream_tokens": call.ctx, "fresh_rows": call.T,
           "steps": steps, "ms_per_step": round(ms, 4), "algorithmic_bytes_per_step": nbytes,
           "value": round(nbytes / ms / 1e6, 1), "unit": "GB/s", "frac": round(nbytes / ms / 1e6 / peak, 4),
           "per_op": timer.per_op(call, peak)}
    del group, inputs, ind, meta
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------------------------------ CPU baseline

def cpu_baseline(call, layers, budget_s, seed):
    """The C oracle (a port of the reference's glue math) on the host cores: a bounded sample of the
    same call -- layers of the workload taken in order until `budget_s` of CPU time is spent."""
    from glmkv import traffic
    from glmkv import workload as W
    from glmkv.stage import FULL
    from oracle import cpu

    sys.path.insert(0, str(ROOT / "tests"))
    from layer_case import LayerCase, run_oracle

    cores = len(os.sched_getaffinity(0))
    cpu.set_threads(cores)
    case = LayerCase(call, "fp8", seed=seed, with_topk=True)
    done, nbytes, elapsed = [], 0, 0.0
    h = case.host()
    while elapsed < budget_s:  # the layers in order, again from the first while budget is left
        for l in layers:
            full = l in FULL
            t0 = time.perf_counter()
            run_oracle(case, h, full)
            elapsed += time.perf_counter() - t0
            nbytes += traffic.layer(call.T, call.ctx, full) + traffic.plan(call.T, call.nseq)
            done.append(l)
            if elapsed >= budget_s:
                break
    return {"value": nbytes / elapsed / 1e9, "unit": "GB/s", "cores": cpu.threads(), "kind": "port",
            "sample": f"{len(done)} layer passes of the workload's layers in order (same call, one layer's "
                      f"cache state reused), {elapsed:.1f} s of C-oracle time, OpenMP over rows / pages",
            "tokens_per_s": call.T / (elapsed / len(done) * len(layers))}


# ------------------------------------------------------------------------------------------ main

def main():
    a = parse()
    import torch

    from glmkv import dist as gd, stage, traffic, workload as W

    world, rank, local = gd.env()
    if world != a.gpus:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE {world}")

    call = W.config(a.workload, seed=a.seed)
    any_layer = a.placement == "any"
    if a.workload == "cfg3":
        if a.cuts:
            cuts = [int(x) for x in a.cuts.split(",")]
            if len(cuts) != world or cuts[0] != 0 or cuts != sorted(set(cuts)) or cuts[-1] >= stage.LAYERS:
                raise SystemExit(f"--cuts {a.cuts}: {world} increasing first layers from 0 below {stage.LAYERS}")
        else:
            cuts = list(stage.cuts(world, T=call.T, ctx=call.ctx, any_layer=any_layer))
        first, last = (cuts + [stage.LAYERS])[rank], (cuts + [stage.LAYERS])[rank + 1]
    else:  # single-layer workloads: every rank runs layer 0 (an indexer layer) of its own call
        first, last, cuts = 0, 1, [0]
    forwards = stage.forwarded_picks(cuts) if a.workload == "cfg3" else []

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    gd.init("nccl", timeout_s=300, device=dev)
    if a.impl == "reference":
        from oracle import ref
        if not ref.available():
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable":
                                  "oracle/_ref/libglmref.so was not built (the reference tree was absent at build time)"}))
            return

    group = stage.LayerGroup(first, last, n_pages=call.n_pages, max_ctx=max(call.ctx, 1), chunk=call.T, device=dev)
    gen = torch.Generator(device=dev).manual_seed(1000 * a.seed + rank)
    group.rope = torch.from_numpy(W.rope_table(int(call.seq_lens.max())).view(np.int16)).to(dev).view(torch.bfloat16)
    fill_caches(torch, group, gen)
    inputs = layer_inputs(torch, group, call.T, gen)
    ind = topk_picks(torch, call, group, gen)
    meta = device_call(torch, call, dev)
    torch.cuda.synchronize()

    # the picks of an indexer layer before a cut at a shared layer travel to the next stage every call
    fwd = gd.picks_forwarder(cuts if a.workload == "cfg3" else [0], rank, call.T, dev, ind=ind, tlen=group.tlen)
    if a.impl == "glmkv":
        call_path = lambda hook: group.run_call(meta, inputs, ind, on_op=hook)
    else:
        call_path = lambda hook: run_call_reference(group, meta, inputs, ind, call.ctx, on_op=hook)

    def run(hook=None):
        fwd.begin_call()
        call_path(compose(fwd.hook if fwd.active else None, hook))
        fwd.end_call()
    launches_per_step = group.launches_per_call()

    barrier = gd.barrier
    max_over_ranks = lambda v: gd.max_over_ranks(v, device=dev)
    uuids = gd.gather_objects(str(getattr(torch.cuda.get_device_properties(dev), "uuid", "")))
    ids = [u if u.startswith("GPU-") else f"GPU-{u}" for u in uuids if u]

    # ---- device-resident timing
    for _ in range(a.warmup):
        run()
    fwd.drain()
    torch.cuda.synchronize()
    barrier()
    # per-kernel timing inside the timed region: events around every kernel of one layer a step (a
    # different layer each step) and around the stage's row plan, on the launch stream
    timer = OpTimer(torch)
    layers = group.layers

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(ids, enabled=(rank == 0 and not a.no_clocks)) as clk:
        torch.cuda.synchronize()
        barrier()
        start.record()
        for i in range(a.steps):
            timer.target = layers[i % len(layers)]
            run(timer)
        fwd.drain()
        end.record()
        torch.cuda.synchronize()
        barrier()
    ms = start.elapsed_time(end)
    ms_max = max_over_ranks(ms)
    rank_ms = gd.gather_objects(round(ms / a.steps, 4))
    dq_us = timer.mean_us("kv_dequant")
    dq_launches = len(timer.spans.get("kv_dequant", []))

    # ---- end to end through the public API: metadata from pinned host memory in, tlen out
    e2e = None
    if not a.no_e2e:
        host = {k: getattr(meta, k).cpu().pin_memory() for k in ("cu", "seq_lens", "block_table", "slot")}
        out = torch.empty(call.T, dtype=torch.int32).pin_memory()
        h2d = sum(v.numel() * v.element_size() for v in host.values())
        d2h = out.numel() * out.element_size()

        def e2e_step():
            for k, v in host.items():
                getattr(meta, k).copy_(v, non_blocking=True)
            run()
            out.copy_(group.tlen[:call.T], non_blocking=True)

        for _ in range(max(1, a.warmup // 2)):
            e2e_step()
        fwd.drain()
        torch.cuda.synchronize()
        barrier()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        s2.record()
        for _ in range(a.steps):
            e2e_step()
        fwd.drain()
        e2.record()
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) * 1e3
        barrier()
        e2e_ms = max_over_ranks(max(s2.elapsed_time(e2), 0.0))
        e2e = (e2e_ms, h2d, d2h, max_over_ranks(wall))

    # the last call that moves picks is done: unmap the peers' buffers on every rank before any rank
    # goes on (ranks other than 0 exit below, which frees the buffers they exported)
    fwd.close()
    barrier()

    # ---- whole-job numbers
    layer_ranges = list(zip(cuts, cuts[1:] + [stage.LAYERS if a.workload == "cfg3" else 1]))
    total_bytes = 0
    for f, l in (layer_ranges if a.workload == "cfg3" else [(0, 1)] * world):
        total_bytes += traffic.plan(call.T, call.nseq) + sum(stage.layer_bytes(x, call.T, call.ctx)
                                                             for x in range(f, l))
    step_s = ms_max / a.steps / 1e3
    value = total_bytes / step_s / 1e9
    peak, peak_kind = measured_peak()
    dq_bytes = traffic.kv_dequant(call.ctx)
    dq_avg_s = (dq_us or 0.0) / 1e6
    achieved = dq_bytes / dq_avg_s / 1e9 if dq_launches else None
    launches_total = int(gd.sum_over_ranks(launches_per_step * a.steps, device=dev))

    traffic_rec = None
    tp = ROOT / "profiles" / "ncu_traffic.json"
    if tp.exists() and a.impl == "glmkv":
        try:
            rec = json.loads(tp.read_text()).get("glm_kv_dequant")
            if rec:
                traffic_rec = round(rec["dram_bytes_per_stream_token"] * call.ctx)
        except (ValueError, KeyError):
            traffic_rec = None

    if rank != 0:
        gd.finish()
        return

    forwarder = type(fwd).__name__  # every rank builds the same kind (picks_forwarder decides together)
    if a.workload == "cfg3":
        cost = [sum(stage.layer_bytes(x, call.T, call.ctx) for x in range(f, l)) for f, l in layer_ranges]
        ideal = sum(stage.layer_bytes(x, call.T, call.ctx) for x in range(stage.LAYERS)) / max(cost)
    else:
        ideal = float(world)
    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": a.steps,
        "warmup": a.warmup,
        "ms_per_step": round(ms_max / a.steps, 4),
        "rank_ms_per_step": rank_ms,
        "higher_is_better": True,
        "scaling": "strong" if a.workload == "cfg3" else "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded numpy / torch generators; no dataset or checkpoint)",
        "impl": a.impl,
        "config": {
            "workload": WORKLOADS[a.workload], "seed": a.seed, "fresh_rows": call.T, "seqs": call.nseq,
            "stream_tokens": call.ctx, "kv_cache": "fp8_ds_mla (656 B/token) + indexer 132 B/token",
            "layers": (stage.LAYERS if a.workload == "cfg3" else world), "stage_cuts": cuts,
            "placement": ("cuts at indexer layers only" if not forwards else
                          "cuts at any layer; the picks of the indexer layer before each cut at a shared layer "
                          "are forwarded to the next stage every call, one call ahead (" + (
                              "copy-engine peer copies through CUDA IPC, ordered by stream memory operations"
                              if forwarder == "PeerCopyForwarder" else "NCCL send/recv on a side stream") + ")"),
            "forwarded_picks": [{"from_rank": s_, "to_rank": r_, "indexer_layer": l_,
                                 "bytes_per_call": stage.picks_bytes(call.T)} for s_, r_, l_ in forwards],
            "forwarder": forwarder if forwards else None,
            "parallelism": f"layer groups x{world} (pipeline stages)" + (
                f", {len(forwards)} forward(s) of the picks a call by " + (
                    "copy-engine peer copies" if forwarder == "PeerCopyForwarder" else "NCCL send/recv")
                if forwards else ", no collective on the data path"),
            "l2": "no flush: every layer's cache pool and stream exceed the 126 MB L2",
            "storage": "e4m3 codes + f32 scales in, bf16 out; f32 arithmetic",
        },
        "tokens_per_s": round(call.T / step_s, 1),
        "pct_hbm_peak": {"of_measured": round(value / (world * peak), 4), "of_nominal_8TBs": round(
            value / (world * NOMINAL_HBM_GBS), 4), "measured_peak_gbs": peak, "peak_kind": peak_kind},
        "ideal_speedup_vs_1gpu": round(ideal, 3),
        "roofline": {"kernel": "glm_kv_dequant", "bound": "hbm", "achieved": round(achieved, 1) if achieved else None,
                     "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4) if achieved else None,
                     "traffic": traffic_rec,
                     "traffic_source": "recorded, not captured in this run: ncu dram__bytes_read.sum + "
                                       "dram__bytes_write.sum of one full-size launch (profiles/ncu_traffic.json), "
                                       "per stream token, times this call's stream tokens" if traffic_rec else None,
                     "algorithmic_bytes_per_launch": dq_bytes,
                     "avg_launch_us": round(dq_avg_s * 1e6, 2), "launches_timed": dq_launches,
                     "peak_note": f"{peak_kind} HBM copy bandwidth (MEASURED_PEAKS.json hbm_gbs)"},
        "gpu_launches": launches_total,
        "clocks": clk.summary(),
        "per_op": {
            "note": f"algorithmic bytes per launch over CUDA-event time, fraction of the {peak_kind} HBM peak. "
                    "in_step: events around every kernel of one layer a step inside the timed steps (these "
                    "launches lose the PDL overlap with their neighbours and pay the write-back of the previous "
                    "kernel's dirty L2 lines); isolated: each kernel back to back over the stage's layers after "
                    "the timed steps",
            "in_step": timer.per_op(call, peak),
            "isolated": isolated_ops(torch, a.impl, group, meta, inputs, ind, call, peak)},
    }
    if e2e is not None:
        e2e_ms, h2d, d2h, wall = e2e
        line["e2e"] = {"value": round(total_bytes / (e2e_ms / a.steps / 1e3) / 1e9, 1), "unit": "GB/s",
                       "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                       "ms_per_step": round(e2e_ms / a.steps, 4), "wall_ms_per_step": round(wall / a.steps, 4),
                       "tokens_per_s": round(call.T / (e2e_ms / a.steps / 1e3), 1),
                       "path": "glmkv LayerGroup.run_call (ctypes -> libglmkv.so) with the call's cu_seqlens, "
                               "seq_lens, block_table, slot_mapping copied from pinned host memory each step and "
                               "tlen read back" if a.impl == "glmkv" else
                               "reference kernels (oracle/_ref) with the same host copies"}
    if a.workload == "cfg3" and not a.no_marked:
        line["marked_lift"] = marked_block(torch, a.impl, group, meta, call, dev, peak)
    if world == 1 and a.workload == "cfg3" and not a.no_cfg2:
        line["cfg2"] = cfg2_block(torch, a.impl, dev, a.seed, peak)
    if not a.no_next_rows:
        line["next_rows"] = next_rows(torch, a.impl, call.T, dev)
        line["next_rows"]["glm_mqa_logits_paged"] = mqa_row(torch, a.impl, group, meta, call, dev)
        line["next_rows"]["bf16_cache_path"] = bf16_rows(torch, a.impl, group, meta, call, dev)
    if a.impl == "reference":
        line["cpu_baseline"] = {"value": line["value"], "unit": "GB/s", "cores": 1, "kind": "reference",
                                "sample": "the whole workload: the reference's glue kernels (kern-glm53 "
                                          "source/glm_glue.cu, unmodified, compiled for sm_100a) on the GPU; the "
                                          "reference has no CPU path"}
    elif world == 1 and not a.no_cpu_baseline:
        layers = list(range(first, last))
        line["cpu_baseline"] = cpu_baseline(call, layers, a.cpu_seconds, a.seed)
    print(json.dumps(line), flush=True)
    gd.finish()


if __name__ == "__main__":
    main()
