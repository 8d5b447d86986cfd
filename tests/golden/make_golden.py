"""Golden vectors of the REFERENCE glue kernels, to pin the C oracle on machines without a GPU.

Runs kern-glm53 ``source/glm_glue.cu`` (compiled from source for sm_100a into ``oracle/_ref``) on
seeded inputs from ``glmkv.workload`` and stores its outputs under ``tests/golden/``:

* ``ref_small_<case>.npz``: one layer of a small call -- every output, with the caches reduced to the
  rows this call wrote (the rest of each pool is the seeded input);
* ``ref_digests.json``: for larger calls, SHA-256 of each output that does not depend on rsqrtf
  (plan, row plan, and the prefix rows of the gathered / dequantized streams), and of the inputs, so a
  CPU run can tell generator drift from an oracle mismatch.

Needs a CUDA device and ``oracle/_ref/libglmref.so``:

    python tests/golden/make_golden.py [--out tests/golden]
"""
import argparse
import hashlib
import json
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path[:0] = [str(ROOT), str(ROOT / "kern-glm53_b200"), str(ROOT / "tests")]

from glmkv import workload as W  # noqa: E402
from layer_case import LayerCase, norm_case, q_post_case, quant_case, run_reference, to_host  # noqa: E402

# (name, call config, call seed, case seed, kv dtype, full layer, zero tiles)
SMALL = [
    ("fp8_full", "small", 21, 22, "fp8", True, 2),
    ("fp8_shared", "small", 21, 23, "fp8", False, 0),
    ("bf16_full", "small", 24, 25, "bf16", True, 2),
]
DIGEST = [
    ("cfg0_fp8_full", "cfg0", 3, 11, "fp8", True, 0),
    ("cfg4_fp8_full", "cfg4", 3, 11, "fp8", True, 4),
    ("cfg4_bf16_full", "cfg4", 3, 11, "bf16", True, 4),
    ("cfg1_fp8_full", "cfg1", 3, 11, "fp8", True, 16),
]
EXACT = ("pos", "ks", "ke", "klen", "row_seq", "zero", "ind", "tlen")
Q_POST = [("q_post_full", 512, 41, True), ("q_post_shared", 512, 42, False)]  # (name, rows, seed, full)
NORM_SMALL = [("norm_add", 8, 51, True), ("norm_noadd", 8, 52, False)]  # (name, rows, seed, with a)
QUANT = [("quant_640", 37, 640, 648), ("quant_16384", 512, 16384, 16384)]  # (name, rows, K, ldx)


def small_call(seed):
    """Three short sequences: a prefix with a ragged fresh chunk, an empty prefix, a one-token chunk."""
    rng = np.random.default_rng(seed)
    return W.make_call([100, 0, 129], [40, 23, 1], rng, max_pages=8, spare_pages=3, name="small", seed=seed)


def call_of(cfg, seed):
    return small_call(seed) if cfg == "small" else W.config(cfg, seed=seed)


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def input_digest(case):
    h = hashlib.sha256()
    for a in (case.x, case.rope, case.w.g_q, case.w.g_kv, case.w.ik_w, case.w.ik_b, case.kv_pool, case.idx_pool,
              case.call.block_table, case.call.slot_mapping, case.call.seq_lens, case.call.cu):
        h.update(np.ascontiguousarray(a).tobytes())
    if case.ind is not None:
        h.update(case.ind.tobytes())
    return h.hexdigest()


def prefix_rows(call):
    """Stream rows that hold prefix tokens (written before this call, so independent of its append)."""
    goff = np.concatenate([[0], np.cumsum(call.seq_lens.astype(np.int64))[:-1]])
    return np.concatenate([g + np.arange(p, dtype=np.int64) for g, p in zip(goff, call.prefix)])


def fresh_cache_rows(case, res):
    """The cache rows this call wrote: latent rows and indexer (keys, scale) at its slots."""
    slots = case.call.slot_mapping
    row = 656 if case.kv_dtype == "fp8" else 1152
    kv = res["kv"].reshape(-1, row)[slots]
    pages = res["idx"].reshape(-1, 64 * 132)
    keys = np.stack([pages[s // 64, (s % 64) * 128:(s % 64) * 128 + 128] for s in slots])
    scs = np.stack([pages[s // 64, 8192 + 4 * (s % 64):8196 + 4 * (s % 64)] for s in slots])
    return kv, keys, scs


def run_case(torch, spec):
    name, cfg, cseed, seed, kv_dtype, full, zt = spec
    case = LayerCase(call_of(cfg, cseed), kv_dtype=kv_dtype, seed=seed, zero_tiles=zt)
    d = case.device(torch, torch.device("cuda:0"))
    run_reference(case, d, full)
    torch.cuda.synchronize()
    return case, to_host(d, torch)


def q_post_outputs(torch, T, seed, full):
    """glm_q_post of the reference on q_post_case(T, seed): qmla (tails only), iq, wout."""
    from oracle import ref
    c = q_post_case(T, seed)
    dev = torch.device("cuda:0")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    qb, rope, pos, iw = t(c["qb"].view(np.int16)), t(c["rope"].view(np.int16)), t(c["pos"]), t(c["iw"].view(np.int16))
    qmla = torch.zeros(T * 64 * 576, dtype=torch.int16, device=dev)
    iq = torch.zeros(T * 32 * 128, dtype=torch.uint8, device=dev)
    wout = torch.zeros(T * 32, dtype=torch.float32, device=dev)
    p = lambda x: x.data_ptr()
    ref.q_post(p(qb), c["ldb"], p(rope), p(pos), p(qmla), p(iq) if full else None, p(iw) if full else None,
               p(wout) if full else None, int(full), T)
    torch.cuda.synchronize()
    tails = qmla.cpu().numpy().view(np.uint16).reshape(T, 64, 576)[:, :, 512:]
    return c, {"qmla_tails": tails, "iq": iq.cpu().numpy(), "wout": wout.cpu().numpy().view(np.uint32)}


def q_post_input_digest(c):
    h = hashlib.sha256()
    for a in (c["qb"], c["rope"], c["pos"], c["iw"]):
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def norm_outputs(torch, T, seed, with_a):
    """glm_add_rms_quant of the reference on norm_case(T, seed): res after the add, normed, q, sf."""
    from oracle import ref
    a, res, gamma = norm_case(T, seed, with_a)
    dev = torch.device("cuda:0")
    t = lambda x: None if x is None else torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).to(dev)
    da, dres, dg = t(a), t(res), t(gamma)
    normed = torch.zeros(T * 6144, dtype=torch.int16, device=dev)
    q = torch.zeros(T * 6144, dtype=torch.uint8, device=dev)
    sf = torch.zeros(12 * T * 4, dtype=torch.uint8, device=dev)
    p = lambda x: None if x is None else x.data_ptr()
    ref.add_rms_quant(p(da), p(dres), p(dg), p(normed), p(q), p(sf), T, T)
    torch.cuda.synchronize()
    return {"res": dres.cpu().numpy().view(np.uint16), "normed": normed.cpu().numpy().view(np.uint16),
            "q": q.cpu().numpy(), "sf": sf.cpu().numpy()}


def quant_outputs(torch, T, K, ldx):
    from oracle import ref
    x = quant_case(T, K, ldx)
    dev = torch.device("cuda:0")
    dx = torch.from_numpy(x.view(np.int16)).to(dev)
    q = torch.zeros(T * K, dtype=torch.uint8, device=dev)
    sf = torch.zeros((K + 511) // 512 * T * 4, dtype=torch.uint8, device=dev)
    ref.quant(dx.data_ptr(), ldx, q.data_ptr(), sf.data_ptr(), T, K, T)
    torch.cuda.synchronize()
    return x, {"q": q.cpu().numpy(), "sf": sf.cpu().numpy()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(HERE))
    a = ap.parse_args()
    out = pathlib.Path(a.out)
    out.mkdir(parents=True, exist_ok=True)
    import torch

    for spec in SMALL:
        case, res = run_case(torch, spec)
        kv, keys, scs = fresh_cache_rows(case, res)
        keep = {k: v for k, v in res.items() if k not in ("kv", "idx")}
        np.savez_compressed(out / f"ref_small_{spec[0]}.npz", input_sha=np.array(input_digest(case)), kv_fresh=kv,
                            idx_keys_fresh=keys, idx_sc_fresh=scs, **keep)
    digests = {}
    for spec in DIGEST:
        case, res = run_case(torch, spec)
        pr = prefix_rows(case.call)
        dg = {"input_sha": input_digest(case), **{k: sha(res[k]) for k in EXACT if k in res}}
        if case.kv_dtype == "fp8":
            dg["kvd_prefix"] = sha(res["kvd"].reshape(-1, 576)[pr])
        if spec[5]:
            dg["kg_prefix"] = sha(res["kg"].reshape(-1, 128)[pr])
            dg["ksf_prefix"] = sha(res["ksf"][pr])
        digests[spec[0]] = dg
    for name, T, seed, full in Q_POST:
        c, res = q_post_outputs(torch, T, seed, full)
        digests[name] = {"input_sha": q_post_input_digest(c), **{k: sha(v) for k, v in res.items()}}
    for name, T, K, ldx in QUANT:
        x, res = quant_outputs(torch, T, K, ldx)
        digests[name] = {"input_sha": sha(x), **{k: sha(v) for k, v in res.items()}}
    for name, T, seed, with_a in NORM_SMALL:
        np.savez_compressed(out / f"ref_small_{name}.npz", **norm_outputs(torch, T, seed, with_a))
    (out / "ref_digests.json").write_text(json.dumps(digests, indent=1, sort_keys=True) + "\n")
    print("golden vectors written to", out)


if __name__ == "__main__":
    main()
