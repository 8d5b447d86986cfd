"""One layer of the cache path (cfg0, fp8, an indexer layer; plus the marked lift) in a fresh process,
printing a digest of every output and the launch shapes the library reports: run by
tests/test_gpu_switches.py under different launch switches (GLMKV_PDL, GLMKV_RESERVE_SMS)."""
import hashlib
import json
import pathlib
import sys

ROOT = pathlib.Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT), str(ROOT / "kern-glm53_b200"), str(ROOT / "tests")]

import numpy as np  # noqa: E402
import torch  # noqa: E402


def main():
    import glmkv
    from glmkv import workload as W
    from layer_case import LayerCase

    dev = torch.device("cuda:0")
    call = W.config("cfg0", seed=41)
    case = LayerCase(call, "fp8", seed=41, with_topk=True)
    d = case.device(torch, dev)
    c, T = call, call.T
    glmkv.plan(d["cu"], d["seq_lens"], c.nseq, d["pos"], d["ks"], d["ke"], d["klen"], d["row_seq"], d["zero"], T)
    glmkv.mla_prep_full(d["x"], case.lda, d["g_q"], d["g_kv"], d["rope"], d["pos"], d["slot"], d["kv"], d["idx"],
                        d["ik_w"], d["ik_b"], d["qq"], d["qsf"], case.sf_rows, T, kv_dtype="fp8")
    glmkv.idx_gather(d["idx"], d["block_table"], c.max_pages, d["seq_lens"], c.nseq, d["kg"], d["ksf"])
    words = (c.ctx + 63) // 64
    mask = torch.empty(words, dtype=torch.int64, device=dev)
    glmkv.topk_stream_mark(d["ind"], d["ks"], d["klen"], d["tlen"], T, d["ke"], mask, words)
    glmkv.kv_dequant(d["kv"], d["block_table"], c.max_pages, d["seq_lens"], c.nseq, d["kvd"])
    marked = torch.zeros_like(d["kvd"])
    glmkv.kv_dequant_marked(d["kv"], d["block_table"], c.max_pages, d["seq_lens"], c.nseq, mask, marked)
    torch.cuda.synchronize()
    digest = hashlib.sha256()
    for k in ("pos", "ks", "ke", "klen", "row_seq", "qq", "qsf", "kv", "idx", "kg", "ksf", "ind", "tlen", "kvd"):
        digest.update(d[k].contiguous().view(torch.uint8).cpu().numpy().tobytes())
    digest.update(mask.cpu().numpy().tobytes())
    digest.update(marked.view(torch.uint8).cpu().numpy().tobytes())
    # at a prefill chunk's 16,384 rows, where no grid is capped by the call's rows
    shapes = {e: glmkv.launch_shape(e, 16384) for e in ("glm_kv_dequant", "glm_idx_gather", "glm_mla_prep_fp8",
                                                        "glm_mark_rows")}
    print(json.dumps({"digest": digest.hexdigest(), "faults": glmkv.fault_flags(),
                      "sms": torch.cuda.get_device_properties(dev).multi_processor_count, "shapes": shapes}))


if __name__ == "__main__":
    main()
