// Host launchers for the REFERENCE glue kernels (kern-glm53 `source/glm_glue.cu`), compiled from the
// reference's own source file, unmodified, for sm_100a. TEST INFRASTRUCTURE ONLY: the library this
// builds (oracle/_ref/libglmref.so) is the bit-exact oracle the GPU parity tests compare against, and
// the arm `bench.py --impl reference` times. It is never part of the product path.
//
// The reference source is included by path at build time (oracle/build.py passes -I to the reference
// tree); nothing of it is copied into this repository. Each launcher uses the grid and block the
// reference's manifest gives the entry (kern-glm53 scripts/gen.py:95-98, 124-135, 172-177):
//   glm_plan           grid ceil(T / 256), block 256
//   glm_mla_prep{_fp8} grid T,             block 256
//   glm_idx_gather     grid ceil(ctx / 64) + seqs, block 256
//   glm_kv_dequant     grid ceil(ctx / 64) + seqs, block 256
//   glm_topk_stream    grid T,             block 256
//   glm_topk_slots     grid T,             block 256
//   glm_q_post         grid T,             block 256 (gen.py:117-123)
//   glm_add_rms_quant  grid T,             block 256 (gen.py:168-171)
//   glm_quant          grid ceil(T * K / 1024), block 256 (gen.py:103-105)
// `ctx` is the manifest's launch variable (the sum of seq_lens); the caller passes it.
#include <cuda_runtime.h>

#include "glm_glue.cu"

#define REF_API extern "C" __attribute__((visibility("default")))

static int ref_status() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

REF_API int ref_glm_plan(const long long* cu, const int* seq_lens, int nseq, int* pos, unsigned* ks, unsigned* ke,
                         int* klen, int* row_seq, int* zero, int T, void* stream) {
  if (T <= 0) return 0;
  glm_plan<<<(T + 255) / 256, 256, 0, (cudaStream_t)stream>>>(cu, seq_lens, nseq, pos, ks, ke, klen, row_seq, zero, T);
  return ref_status();
}

REF_API int ref_glm_mla_prep(int fp8, const bf16* x, int lda, const bf16* g_q, const bf16* g_kv, const bf16* rope,
                             const int* pos, const long long* slot, u8* kv, u8* idx, const bf16* ik_w, const bf16* ik_b,
                             u8* qq, u8* qsf, int sf_rows, int T, void* stream) {
  if (T <= 0) return 0;
  if (fp8)
    glm_mla_prep_fp8<<<T, 256, 0, (cudaStream_t)stream>>>(x, lda, g_q, g_kv, rope, pos, slot, kv, idx, ik_w, ik_b, qq,
                                                          qsf, sf_rows, T);
  else
    glm_mla_prep<<<T, 256, 0, (cudaStream_t)stream>>>(x, lda, g_q, g_kv, rope, pos, slot, kv, idx, ik_w, ik_b, qq, qsf,
                                                      sf_rows, T);
  return ref_status();
}

REF_API int ref_glm_idx_gather(const u8* idx, const int* block_table, int max_pages, const int* seq_lens, int nseq,
                               u8* kg, float* ksf, int ctx, void* stream) {
  const int grid = (ctx + PAGE - 1) / PAGE + nseq;
  if (grid <= 0) return 0;
  glm_idx_gather<<<grid, 256, 0, (cudaStream_t)stream>>>(idx, block_table, max_pages, seq_lens, nseq, kg, ksf);
  return ref_status();
}

REF_API int ref_glm_kv_dequant(const u8* kv, const int* block_table, int max_pages, const int* seq_lens, int nseq,
                               bf16* kvd, int ctx, void* stream) {
  const int grid = (ctx + PAGE - 1) / PAGE + nseq;
  if (grid <= 0) return 0;
  glm_kv_dequant<<<grid, 256, 0, (cudaStream_t)stream>>>(kv, block_table, max_pages, seq_lens, nseq, kvd);
  return ref_status();
}

REF_API int ref_glm_topk_stream(int* ind, const unsigned* ks, const int* klen, int* tlen, int T, void* stream) {
  if (T <= 0) return 0;
  glm_topk_stream<<<T, 256, 0, (cudaStream_t)stream>>>(ind, ks, klen, tlen, T);
  return ref_status();
}

REF_API int ref_glm_topk_slots(int* ind, const int* block_table, int max_pages, const int* row_seq, const int* klen,
                               int* tlen, int T, void* stream) {
  if (T <= 0) return 0;
  glm_topk_slots<<<T, 256, 0, (cudaStream_t)stream>>>(ind, block_table, max_pages, row_seq, klen, tlen, T);
  return ref_status();
}

REF_API int ref_glm_q_post(const bf16* qb, int ldb, const bf16* rope, const int* pos, bf16* qmla, u8* iq, const bf16* iw,
                           float* wout, int full, int T, void* stream) {
  if (T <= 0) return 0;
  glm_q_post<<<T, 256, 0, (cudaStream_t)stream>>>(qb, ldb, rope, pos, qmla, iq, iw, wout, full, T);
  return ref_status();
}

REF_API int ref_glm_add_rms_quant(const bf16* a, bf16* res, const bf16* gamma, bf16* normed, u8* q, u8* sf, int sf_rows,
                                  int T, void* stream) {
  if (T <= 0) return 0;
  glm_add_rms_quant<<<T, 256, 0, (cudaStream_t)stream>>>(a, res, gamma, normed, q, sf, sf_rows, T);
  return ref_status();
}

REF_API int ref_glm_quant(const bf16* x, int ldx, u8* q, u8* sf, int sf_rows, int K, int T, void* stream) {
  const long long warps = (long long)T * (K >> 7);
  if (warps <= 0) return 0;
  glm_quant<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(x, ldx, q, sf, sf_rows, K, T);
  return ref_status();
}
