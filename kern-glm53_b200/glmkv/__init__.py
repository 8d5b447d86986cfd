"""glmkv: GLM-5.3's prefill KV-cache path on B200 (sm_100a).

Drop-in replacement for the cache ops of kern-glm53's ``source/glm_glue.cu`` (plan, the fp8 / bf16
latent-cache append with the indexer-key append, the indexer-key gather, the paged fp8 -> bf16
dequant, the top-k row plans), with the ops beside it: the q_pe rope and indexer query, the norm and
quant glue, the indexer's MQA logits read straight from the cache pages, and a lift of only the rows
the picks name (mark_rows or topk_stream_mark, kv_dequant_marked). The kernels are CUDA in ``libglmkv.so`` (C ABI: ``include/glmkv.h``);
this package binds them with ctypes and uses PyTorch only to own device memory.
"""
from ._lib import CUBIN_PATH, LIB_PATH, GlmKvError, fault_flags, launch_shape, lib, strerror
from .ops import (add_rms_quant, head_norm, idx_gather, kv_dequant, kv_dequant_marked, mark_rows, mla_prep_full,
                  mla_prep_shared, mqa_logits_paged, plan, q_post_full, q_post_shared, quant_o, rms_quant, topk_slots,
                  topk_stream, topk_stream_mark)

__all__ = ["CUBIN_PATH", "LIB_PATH", "GlmKvError", "fault_flags", "launch_shape", "lib", "strerror", "plan", "mla_prep_full",
           "mla_prep_shared", "idx_gather", "kv_dequant", "topk_stream", "topk_slots", "q_post_full", "q_post_shared",
           "add_rms_quant", "rms_quant", "head_norm", "quant_o", "mqa_logits_paged", "mark_rows", "topk_stream_mark",
           "kv_dequant_marked"]
