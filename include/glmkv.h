/*
 * glmkv: GLM-5.3's prefill KV-cache path for B200 (sm_100a), as a C ABI.
 *
 * Each launcher takes exactly the parameter list of the kern-glm53 manifest op it replaces, in the
 * same order, followed by the CUDA stream to launch on. Pointers are device addresses; bf16 data is
 * passed as `const void*` (16-bit bfloat16 elements), e4m3 as bytes. Nothing is allocated or freed;
 * every launcher only enqueues work on `stream` and is safe to call from several host threads on
 * different streams. The same kernels, with the same entry names and parameter lists, are also built
 * as the cubin `glm_glue_b200.cubin` for a kern manifest.
 *
 * Launches use programmatic dependent launch (unless the environment sets GLMKV_PDL=0): a kernel may
 * start while the kernel before it on the stream drains, and waits for it before it reads anything
 * that kernel can have written. The one exception is the append's norm weights (g_q, g_kv, ik_w,
 * ik_b), load-time constants read before that wait: they must not be written by the kernel launched
 * just before the append. (The append also prefetches its first rows of x into L2 before the wait; a
 * prefetch reads no value into the kernel, so it needs no such condition.)
 *
 * The persistent kernels (append, gather, dequant and its marked form, the marks, add_rms_quant, MQA
 * logits) size their grids for every SM of the device, less GLMKV_RESERVE_SMS when the environment
 * sets it (read once per device, at the first launch): SMs left to other kernels that stay resident
 * beside the path, such as a transfer that waits for its peer.
 *
 * Return value: GLMKV_OK, or a GLMKV_ERR_* code when an argument is invalid (nothing is launched) or
 * the launch failed. Device-side conditions (an invalid page number in a block table, a bounded wait
 * that gave up) are recorded in the module's fault word, read with glmkv_fault_flags().
 *
 * Cache layouts (kern-glm53 source/glm_glue.cu:14-18, scripts/gen.py:53-61), slot s = page s / 64,
 * row s % 64 of both caches:
 *   latent cache, fp8_ds_mla: 656 B a token: 512 e4m3 (four tiles of 128) | 4 x f32 tile scales |
 *                             64 bf16 roped k_pe; a page is 64 x 656 = 41984 B.
 *   latent cache, bf16:       576 bf16 a token (1152 B).
 *   indexer cache:            a page of 64 tokens is 64 x 128 e4m3 keys, then their 64 f32 scales
 *                             (8448 B; 132 B a token).
 */
#ifndef GLMKV_H
#define GLMKV_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct CUstream_st;
typedef struct CUstream_st* glmkv_stream_t; /* a cudaStream_t; NULL is the legacy default stream */

enum {
  GLMKV_OK = 0,
  GLMKV_ERR_ARG = 1,     /* a null pointer where one is required, or a size out of range */
  GLMKV_ERR_ALIGN = 2,   /* a pointer or row stride without the alignment the kernel's accesses need */
  GLMKV_ERR_DEVICE = 3,  /* no usable CUDA device, or the device query failed */
  GLMKV_ERR_LAUNCH = 4   /* the kernel launch failed (cudaGetLastError after the launch) */
};

/* A row's sequence, position and indexer bounds.
 * Replaces op `plan` -> glm_plan (kern-glm53 scripts/gen.py:95-98; source/glm_glue.cu:109-125).
 * cu [nseq + 1] i64 prefix of the call's fresh rows, seq_lens [nseq] i32 (prefix + fresh),
 * outputs [T]: pos, klen, row_seq, zero i32; ks, ke u32. Needs nseq >= 1, T >= 0. */
int glmkv_plan(const int64_t* cu, const int32_t* seq_lens, int nseq, int32_t* pos, uint32_t* ks, uint32_t* ke,
               int32_t* klen, int32_t* row_seq, int32_t* zero, int T, glmkv_stream_t stream);

/* The latent-cache append with the q_a norm + quant, bf16 latent rows (--kv bf16).
 * Replaces ops `mla_prep_full` / `mla_prep_shared` -> glm_mla_prep (kern-glm53 scripts/gen.py:172-177;
 * source/glm_glue.cu:202-296). x [T, lda] bf16: q_a 2048 | kv_a 512 | k_pe 64 | wk 128; rope [pos][64]
 * bf16 (32 cos | 32 sin); slot [T] i64 (< 0: no cache write); idx, ik_w, ik_b all NULL on a shared
 * layer; qq [T, 2048] e4m3 out; qsf DeepGEMM-packed UE8M0 words [(2048 / 512)][sf_rows] out.
 * Needs lda % 4 == 0 and lda >= 2624 (2752 with idx), x, g_q, ik_w and ik_b 8-byte aligned; g_kv,
 * rope, qq, qsf, kv and idx 4-byte aligned (rows of x that are 16-byte aligned, lda % 8 == 0 and x
 * 16-byte aligned, are staged by bulk copies, the others read directly); sf_rows >= T. */
int glmkv_mla_prep(const void* x, int lda, const void* g_q, const void* g_kv, const void* rope, const int32_t* pos,
                   const int64_t* slot, void* kv, void* idx, const void* ik_w, const void* ik_b, void* qq, void* qsf,
                   int sf_rows, int T, glmkv_stream_t stream);

/* The same append into the fp8_ds_mla latent cache (the default --kv fp8).
 * Replaces ops `mla_prep_full` / `mla_prep_shared` -> glm_mla_prep_fp8 (kern-glm53 scripts/gen.py:172-177;
 * source/glm_glue.cu:202-287, 297-299). Same arguments and requirements as glmkv_mla_prep. */
int glmkv_mla_prep_fp8(const void* x, int lda, const void* g_q, const void* g_kv, const void* rope,
                       const int32_t* pos, const int64_t* slot, void* kv, void* idx, const void* ik_w, const void* ik_b,
                       void* qq, void* qsf, int sf_rows, int T, glmkv_stream_t stream);

/* The indexer keys of every sequence gathered back to back into kg [., 128] u8 and ksf [.] f32.
 * Replaces op `idx_gather` -> glm_idx_gather (kern-glm53 scripts/gen.py:124-126;
 * source/glm_glue.cu:357-376). block_table [nseq, max_pages] i32. Needs idx and kg 16-byte aligned. */
int glmkv_idx_gather(const void* idx, const int32_t* block_table, int max_pages, const int32_t* seq_lens, int nseq,
                     void* kg, float* ksf, glmkv_stream_t stream);

/* The fp8 latent rows of every sequence lifted to a contiguous bf16 stream kvd [., 576].
 * Replaces op `kv_dequant` -> glm_kv_dequant (kern-glm53 scripts/gen.py:133-135;
 * source/glm_glue.cu:382-414). Needs kv and kvd 16-byte aligned. */
int glmkv_kv_dequant(const void* kv, const int32_t* block_table, int max_pages, const int32_t* seq_lens, int nseq,
                     void* kvd, glmkv_stream_t stream);

/* The stream rows a call's picks name, as a bitmap for glmkv_kv_dequant_marked: bit p % 64 of word
 * p / 64 of mask is set for every pick p >= 0 of ind [T, 2048] i32 (stream rows: glmkv_topk_stream's
 * output). ks and ke [T] u32 are glm_plan's: row r's picks lie in [ks[r], ke[r]). The launcher first
 * clears mask [mask_words] (one memset on `stream`; mask_words >= ceil(stream rows / 64)). A pick at or
 * past mask_words * 64 is skipped and sets fault bit 4. The shared layers after an indexer layer attend
 * with its picks, so one mask serves them all. Needs ind 16-byte aligned, mask 8.
 * No counterpart in the reference, which lifts every row (kern-glm53 source/glm_glue.cu:378-414). */
int glmkv_mark_rows(const int32_t* ind, const uint32_t* ks, const uint32_t* ke, int T, uint64_t* mask, int mask_words,
                    glmkv_stream_t stream);

/* glmkv_topk_stream and glmkv_mark_rows in one pass over the picks: ind [T, 2048] i32 arrives
 * sequence-relative and leaves as stream rows (in place, the bytes glmkv_topk_stream writes), tlen as
 * glmkv_topk_stream writes it, and mask as glmkv_mark_rows builds it from those stream rows. The first
 * five parameters are glmkv_topk_stream's, the rest glmkv_mark_rows'. Clears mask first, as
 * glmkv_mark_rows does. Needs ind 16-byte aligned, mask 8. No counterpart in the reference: it
 * replaces op `topk_stream` (kern-glm53 scripts/gen.py:130-132; source/glm_glue.cu:416-428) on an
 * indexer layer whose picks the row-selective lift uses. */
int glmkv_topk_stream_mark(int32_t* ind, const uint32_t* ks, const int32_t* klen, int32_t* tlen, int T,
                           const uint32_t* ke, uint64_t* mask, int mask_words, glmkv_stream_t stream);

/* glmkv_kv_dequant restricted to the rows mask marks (glmkv_mark_rows): every marked stream row gets
 * exactly the bytes glmkv_kv_dequant writes there. A page with no marked row is neither read nor
 * written. A page with 48 or more marked rows is lifted whole (its other rows get the bytes
 * glmkv_kv_dequant writes there); of the other pages only the span from the first to the last marked
 * row is read and only the marked rows are written. mask holds ceil(stream rows / 64) words. Needs kv
 * and kvd 16-byte aligned, mask 8.
 * No counterpart in the reference (its op `kv_dequant`, kern-glm53 scripts/gen.py:133-135, lifts every
 * row; FlashMLA reads only the picked rows, scripts/gen.py:399-400). */
int glmkv_kv_dequant_marked(const void* kv, const int32_t* block_table, int max_pages, const int32_t* seq_lens,
                            int nseq, const uint64_t* mask, void* kvd, glmkv_stream_t stream);

/* Top-k picks [T, 2048] i32 (sequence-relative, -1 padded) -> stream rows, in place; tlen [T].
 * Replaces op `topk_stream` -> glm_topk_stream (kern-glm53 scripts/gen.py:130-132;
 * source/glm_glue.cu:419-428). Needs ind 16-byte aligned. */
int glmkv_topk_stream(int32_t* ind, const uint32_t* ks, const int32_t* klen, int32_t* tlen, int T,
                      glmkv_stream_t stream);

/* Top-k picks -> cache slots through the row's page table, in place; tlen [T] (--kv bf16).
 * Replaces op `topk_slots` -> glm_topk_slots (kern-glm53 scripts/gen.py:127-129;
 * source/glm_glue.cu:433-444). Needs ind 16-byte aligned. */
int glmkv_topk_slots(int32_t* ind, const int32_t* block_table, int max_pages, const int32_t* row_seq,
                     const int32_t* klen, int32_t* tlen, int T, glmkv_stream_t stream);

/* After the q_b GEMM: the rope of each head's q_pe into the tail of the absorbed query qmla
 * [T, 64, 576] bf16 and, when `full`, the indexer query: rope on its first 64 dims, e4m3 per
 * (row, head) into iq [T, 32, 128] with a UE8M0 scale, and the head weight
 * wout [T, 32] f32 = ((iw * scale) * 128^-0.5) * 32^-0.5.
 * Replaces ops `q_post_full` / `q_post_shared` -> glm_q_post (kern-glm53 scripts/gen.py:117-123;
 * source/glm_glue.cu:306-351). qb [T, ldb] bf16: 64 heads of nope 192 | pe 64, then 32 indexer heads
 * of 128. iq, iw, wout may be NULL when full == 0. Needs qb and qmla 16-byte aligned, ldb % 8 == 0,
 * rope 8-byte aligned. */
int glmkv_q_post(const void* qb, int ldb, const void* rope, const int32_t* pos, void* qmla, void* iq, const void* iw,
                 float* wout, int full, int T, glmkv_stream_t stream);

/* The residual add + RMSNorm + quant: res = bf16(a + res) written back (a NULL: res is already the
 * stream), normed = bf16(bf16(res * rr) * gamma) with rr = rsqrt(sum(res^2) / 6144 + 1e-5), and normed
 * quantized per 128 columns into q [T, 6144] e4m3 and sf (DeepGEMM-packed UE8M0 words
 * [(6144 / 512)][sf_rows]). Rows are 6144 wide. normed, q (with sf) may be NULL.
 * Replaces ops `add_rms_quant`, `rms_quant` (a NULL), `head_norm` (q, sf NULL) -> glm_add_rms_quant
 * (kern-glm53 scripts/gen.py:156-158, 168-171; source/glm_glue.cu:127-162). Needs res and a 16-byte
 * aligned, gamma and normed 8, q 4, sf_rows >= T when q is given. */
int glmkv_add_rms_quant(const void* a, void* res, const void* gamma, void* normed, void* q, void* sf, int sf_rows,
                        int T, glmkv_stream_t stream);

/* x [T, K] bf16 (rows ldx apart) quantized per 128 columns into q [T, K] e4m3 and sf.
 * Replaces op `quant_o` -> glm_quant (kern-glm53 scripts/gen.py:103-105; source/glm_glue.cu:164-175).
 * Needs K % 128 == 0, ldx >= K, ldx % 8 == 0, x and q 16-byte aligned, sf 4, sf_rows >= T. */
int glmkv_quant(const void* x, int ldx, void* q, void* sf, int sf_rows, int K, int T, glmkv_stream_t stream);

/* The indexer's fp8 MQA logits read straight from the indexer cache pages (the gather-free input
 * format): for each row r < R and key position p < klen[r] of its sequence row_seq[r],
 *   logits[r * stride + p] = sum_h w[r][h] * relu(sum_d iq[r][h][d] * key[p][d]) * scale[p],
 * key / scale at page block_table[row_seq[r] * max_pages + p / 64], row p % 64 of `idx` (n_pages
 * pages of 8448 B). Positions p >= klen[r] (or >= stride) are not written.
 * Replaces ops `idx_gather` plus the indexer's MQA launch (kern-glm53 scripts/gen.py:124-126,
 * scripts/glm_ops.py:104-134: DeepGEMM's sm100 fp8 MQA logits on the gathered kg / ksf, compressed
 * layout). iq [R, 32, 128] e4m3 and w [R, 32] f32 are glm_q_post's iq and wout; row_seq and klen come
 * from glm_plan. Runs on the tensor cores (tcgen05, kind::f8f6f4). Needs iq, idx and w 16-byte aligned,
 * logits 4-byte aligned, stride >= every klen. */
int glmkv_mqa_logits_paged(const void* iq, const void* idx, int n_pages, const int32_t* block_table, int max_pages,
                           const int32_t* row_seq, const int32_t* klen, const float* w, float* logits, int stride,
                           int R, glmkv_stream_t stream);

/* The launch shape (grid x, block x, dynamic shared memory bytes) libglmkv uses for the kernel
 * `entry` ("glm_plan", "glm_mla_prep", "glm_mla_prep_fp8", "glm_idx_gather", "glm_kv_dequant",
 * "glm_topk_stream", "glm_topk_slots", "glm_q_post", "glm_add_rms_quant", "glm_mqa_logits_paged",
 * "glm_mark_rows", "glm_topk_stream_mark", "glm_kv_dequant_marked") on the current device for a
 * call of T fresh rows: what a kern
 * manifest's `impl.launches` entry for the cubin must use. The persistent page kernels depend on the
 * device's SM count only. No counterpart in the reference, whose shapes are fixed in its manifest
 * generator (kern-glm53 scripts/gen.py:95-135, 172-177). */
int glmkv_launch_shape(const char* entry, int T, int* grid, int* block, int* smem_bytes);

/* Self-test of the bounded wait the page pipelines use: a kernel waits on a barrier that nothing
 * completes, gives up after `limit_ns` (at most one second), sets fault bit 1 and writes the time it
 * waited to the device word `waited_ns`. Lets a test check the timeout path without a fault. No
 * counterpart in the reference. */
int glmkv_selftest_wait(uint64_t limit_ns, uint32_t* waited_ns, glmkv_stream_t stream);

/* Device-side fault bits of the current device's module (1: a bounded wait gave up; 2: a block
 * table named a negative page, which was skipped; 4: a pick past the mark bitmap, skipped). Synchronises the device; clears the word when
 * `clear` is non-zero. No counterpart in the reference, whose kernels report nothing. */
int glmkv_fault_flags(uint32_t* flags, int clear);

/* A static description of an error code. */
const char* glmkv_strerror(int code);

/* ABI version of this header (major * 100 + minor). */
int glmkv_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GLMKV_H */
