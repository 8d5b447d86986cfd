// Host side of libglmkv.so: the C ABI of include/glmkv.h. Each launcher validates its arguments on
// the host (returning before any CUDA call when they are invalid), picks the launch shape and
// enqueues one kernel on the caller's stream. No allocation, no synchronisation.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include <cudaTypedefs.h>

#include "glmkv.h"
#include "glmkv_kernels.cuh"
#include "glmkv_mqa.cuh"

#define GLMKV_API extern "C" __attribute__((visibility("default")))

namespace {

using namespace glmkv;

constexpr int MAX_DEVICES = 64;
constexpr size_t DQ_SMEM = (size_t)DQ_STAGES * KV8_PAGE;
constexpr size_t GA_SMEM = (size_t)GA_STAGES * IDX_PAGE;

struct DeviceInfo {
  int status = GLMKV_OK;
  int sms = 0;        // SMs the persistent grids are sized for: the device's, less GLMKV_RESERVE_SMS
  int dq_ctas = 0;    // resident dequant CTAs an SM
  int ga_ctas = 0;    // resident gather CTAs an SM
  int prep_ctas = 0;  // resident append CTAs an SM
  int arq_ctas = 0;   // resident add_rms_quant CTAs an SM
  int mq_ctas = 0;    // resident MQA logits CTAs an SM
};

std::once_flag g_once[MAX_DEVICES];
DeviceInfo g_info[MAX_DEVICES];

// Per device, once: opt the page pipelines into their shared memory, and size their persistent grids.
const DeviceInfo* device_info() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) {
    cudaGetLastError();
    return nullptr;
  }
  std::call_once(g_once[dev], [dev] {
    DeviceInfo& d = g_info[dev];
    bool ok = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess;
    // SMs left to other work that runs beside the path on the same GPU, such as a transfer kernel that
    // stays resident while it waits for its peer: a persistent grid sized for every SM would otherwise
    // have a CTA wait for that kernel, and the whole launch with it
    if (const char* r = getenv("GLMKV_RESERVE_SMS")) {
      const int reserve = atoi(r);
      if (reserve > 0) d.sms = std::max(1, d.sms - reserve);
    }
    ok = ok && cudaFuncSetAttribute(glm_kv_dequant, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)DQ_SMEM) ==
                   cudaSuccess;
    ok = ok && cudaFuncSetAttribute(glm_idx_gather, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GA_SMEM) ==
                   cudaSuccess;
    ok = ok && cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.dq_ctas, glm_kv_dequant, DQ_THREADS, DQ_SMEM) ==
                   cudaSuccess;
    ok = ok && cudaFuncSetAttribute(glm_kv_dequant_marked, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)DQ_SMEM) == cudaSuccess;
    ok = ok && cudaFuncSetAttribute(glm_mark_rows, cudaFuncAttributeMaxDynamicSharedMemorySize, MK_SMEM) ==
                   cudaSuccess;
    ok = ok && cudaFuncSetAttribute(glm_topk_stream_mark, cudaFuncAttributeMaxDynamicSharedMemorySize, MK_SMEM) ==
                   cudaSuccess;
    ok = ok && cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.ga_ctas, glm_idx_gather, GA_THREADS, GA_SMEM) ==
                   cudaSuccess;
    for (auto k : {glm_mla_prep, glm_mla_prep_fp8})
      ok = ok && cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, PREP_SMEM) == cudaSuccess;
    ok = ok && cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.prep_ctas, glm_mla_prep_fp8, PREP_THREADS,
                                                             PREP_SMEM) == cudaSuccess;
    ok = ok && cudaFuncSetAttribute(glm_add_rms_quant, cudaFuncAttributeMaxDynamicSharedMemorySize, ARQ_SMEM) ==
                   cudaSuccess;
    ok = ok && cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.arq_ctas, glm_add_rms_quant, ARQ_THREADS, ARQ_SMEM) ==
                   cudaSuccess;
    ok = ok && cudaFuncSetAttribute(glm_mqa_logits_paged, cudaFuncAttributeMaxDynamicSharedMemorySize, MQ_SMEM) ==
                   cudaSuccess;
    ok = ok && cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.mq_ctas, glm_mqa_logits_paged, MQ_THREADS, MQ_SMEM) ==
                   cudaSuccess;
    if (!ok || d.sms <= 0 || d.dq_ctas <= 0 || d.ga_ctas <= 0 || d.prep_ctas <= 0 || d.arq_ctas <= 0 ||
        d.mq_ctas <= 0) {
      d.status = GLMKV_ERR_DEVICE;
      cudaGetLastError();
    }
  });
  return g_info[dev].status == GLMKV_OK ? &g_info[dev] : nullptr;
}

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Launches use programmatic stream serialization (PDL) unless GLMKV_PDL=0: every kernel waits in
// pdl_wait() before its first global-memory access, so it may be scheduled while the previous kernel
// on the stream drains, which hides the launch latency between the path's back-to-back kernels.
bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("GLMKV_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
int launch(void (*kernel)(KArgs...), int grid, int block, size_t smem, glmkv_stream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...) != cudaSuccess) {
    cudaGetLastError();
    return GLMKV_ERR_LAUNCH;
  }
  return GLMKV_OK;
}

template <bool FP8>
int prep(const void* x, int lda, const void* g_q, const void* g_kv, const void* rope, const int32_t* pos,
         const int64_t* slot, void* kv, void* idx, const void* ik_w, const void* ik_b, void* qq, void* qsf, int sf_rows,
         int T, glmkv_stream_t stream) {
  if (T < 0) return GLMKV_ERR_ARG;
  if (T == 0) return GLMKV_OK;
  if (!x || !g_q || !g_kv || !rope || !pos || !slot || !kv || !qq || !qsf) return GLMKV_ERR_ARG;
  if (idx && (!ik_w || !ik_b)) return GLMKV_ERR_ARG;
  if (lda < (idx ? QL + MLA + ID : QL + MLA) || sf_rows < T) return GLMKV_ERR_ARG;
  if (lda % 4 || !aligned(x, 8) || !aligned(g_q, 8) || !aligned(g_kv, 4) || !aligned(rope, 4) || !aligned(qq, 4) ||
      !aligned(qsf, 4) || !aligned(kv, 4) || (idx && (!aligned(idx, 4) || !aligned(ik_w, 8) || !aligned(ik_b, 8))))
    return GLMKV_ERR_ALIGN;
  const DeviceInfo* d = device_info();
  if (!d) return GLMKV_ERR_DEVICE;
  const int grid = std::min(d->sms * d->prep_ctas, (T + PREP_WARPS - 1) / PREP_WARPS);
  return launch(FP8 ? glm_mla_prep_fp8 : glm_mla_prep, grid, PREP_THREADS, PREP_SMEM, stream, (const bf16*)x, lda,
                (const bf16*)g_q, (const bf16*)g_kv, (const bf16*)rope, pos, (const long long*)slot, (u8*)kv, (u8*)idx,
                (const bf16*)ik_w, (const bf16*)ik_b, (u8*)qq, (u8*)qsf, sf_rows, T);
}

// cuTensorMapEncodeTiled, from the driver through the runtime (no link against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      f = nullptr;
    }
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }();
  return fn;
}

}  // namespace

GLMKV_API int glmkv_plan(const int64_t* cu, const int32_t* seq_lens, int nseq, int32_t* pos, uint32_t* ks,
                         uint32_t* ke, int32_t* klen, int32_t* row_seq, int32_t* zero, int T, glmkv_stream_t stream) {
  if (T < 0 || nseq < 1) return GLMKV_ERR_ARG;
  if (T == 0) return GLMKV_OK;
  if (!cu || !seq_lens || !pos || !ks || !ke || !klen || !row_seq || !zero) return GLMKV_ERR_ARG;
  return launch(glm_plan, (T + PLAN_THREADS - 1) / PLAN_THREADS, PLAN_THREADS, 0, stream, (const long long*)cu, seq_lens,
                nseq, pos, ks, ke, klen, row_seq, zero, T);
}

GLMKV_API int glmkv_mla_prep(const void* x, int lda, const void* g_q, const void* g_kv, const void* rope,
                             const int32_t* pos, const int64_t* slot, void* kv, void* idx, const void* ik_w,
                             const void* ik_b, void* qq, void* qsf, int sf_rows, int T, glmkv_stream_t stream) {
  return prep<false>(x, lda, g_q, g_kv, rope, pos, slot, kv, idx, ik_w, ik_b, qq, qsf, sf_rows, T, stream);
}

GLMKV_API int glmkv_mla_prep_fp8(const void* x, int lda, const void* g_q, const void* g_kv, const void* rope,
                                 const int32_t* pos, const int64_t* slot, void* kv, void* idx, const void* ik_w,
                                 const void* ik_b, void* qq, void* qsf, int sf_rows, int T, glmkv_stream_t stream) {
  return prep<true>(x, lda, g_q, g_kv, rope, pos, slot, kv, idx, ik_w, ik_b, qq, qsf, sf_rows, T, stream);
}

GLMKV_API int glmkv_idx_gather(const void* idx, const int32_t* block_table, int max_pages, const int32_t* seq_lens,
                               int nseq, void* kg, float* ksf, glmkv_stream_t stream) {
  if (nseq < 0 || max_pages < 0) return GLMKV_ERR_ARG;
  if (nseq == 0) return GLMKV_OK;
  if (!idx || !block_table || !seq_lens || !kg || !ksf) return GLMKV_ERR_ARG;
  if (!aligned(idx, 16) || !aligned(kg, 16) || !aligned(ksf, 4)) return GLMKV_ERR_ALIGN;
  const DeviceInfo* d = device_info();
  if (!d) return GLMKV_ERR_DEVICE;
  return launch(glm_idx_gather, d->sms * d->ga_ctas, GA_THREADS, GA_SMEM, stream, (const u8*)idx, block_table,
                max_pages, seq_lens, nseq, (u8*)kg, ksf);
}

GLMKV_API int glmkv_kv_dequant(const void* kv, const int32_t* block_table, int max_pages, const int32_t* seq_lens,
                               int nseq, void* kvd, glmkv_stream_t stream) {
  if (nseq < 0 || max_pages < 0) return GLMKV_ERR_ARG;
  if (nseq == 0) return GLMKV_OK;
  if (!kv || !block_table || !seq_lens || !kvd) return GLMKV_ERR_ARG;
  if (!aligned(kv, 16) || !aligned(kvd, 16)) return GLMKV_ERR_ALIGN;
  const DeviceInfo* d = device_info();
  if (!d) return GLMKV_ERR_DEVICE;
  return launch(glm_kv_dequant, d->sms * d->dq_ctas, DQ_THREADS, DQ_SMEM, stream, (const u8*)kv, block_table,
                max_pages, seq_lens, nseq, (bf16*)kvd);
}

// The checks and the clearing memset of the two marking launchers; GLMKV_OK with *go set when a
// launch of `grid` CTAs follows.
static int mark_prologue(const void* ind, const void* ks, const void* ke, int T, uint64_t* mask, int mask_words,
                         glmkv_stream_t stream, bool* go, int* grid) {
  *go = false;
  if (T < 0 || mask_words < 0) return GLMKV_ERR_ARG;
  if (mask_words == 0) return T == 0 ? GLMKV_OK : GLMKV_ERR_ARG;
  if (!mask) return GLMKV_ERR_ARG;
  if (!aligned(mask, 8)) return GLMKV_ERR_ALIGN;
  if (T > 0 && (!ind || !ks || !ke)) return GLMKV_ERR_ARG;
  if (T > 0 && !aligned(ind, 16)) return GLMKV_ERR_ALIGN;
  const DeviceInfo* d = device_info();
  if (!d) return GLMKV_ERR_DEVICE;
  if (cudaMemsetAsync(mask, 0, (size_t)mask_words * 8, (cudaStream_t)stream) != cudaSuccess) {
    cudaGetLastError();
    return GLMKV_ERR_LAUNCH;
  }
  *go = T > 0;
  *grid = std::min(d->sms, (T + MK_RB - 1) / MK_RB);
  return GLMKV_OK;
}

GLMKV_API int glmkv_mark_rows(const int32_t* ind, const uint32_t* ks, const uint32_t* ke, int T, uint64_t* mask,
                              int mask_words, glmkv_stream_t stream) {
  bool go;
  int grid = 0;
  const int rc = mark_prologue(ind, ks, ke, T, mask, mask_words, stream, &go, &grid);
  if (rc != GLMKV_OK || !go) return rc;
  return launch(glm_mark_rows, grid, MK_THREADS, MK_SMEM, stream, (const int*)ind, (const unsigned*)ks,
                (const unsigned*)ke, T, (unsigned long long*)mask, mask_words);
}

GLMKV_API int glmkv_topk_stream_mark(int32_t* ind, const uint32_t* ks, const int32_t* klen, int32_t* tlen, int T,
                                     const uint32_t* ke, uint64_t* mask, int mask_words, glmkv_stream_t stream) {
  if (T > 0 && (!klen || !tlen)) return GLMKV_ERR_ARG;
  bool go;
  int grid = 0;
  const int rc = mark_prologue(ind, ks, ke, T, mask, mask_words, stream, &go, &grid);
  if (rc != GLMKV_OK || !go) return rc;
  return launch(glm_topk_stream_mark, grid, MK_THREADS, MK_SMEM, stream, (int*)ind, (const unsigned*)ks,
                (const int*)klen, (int*)tlen, T, (const unsigned*)ke, (unsigned long long*)mask, mask_words);
}

GLMKV_API int glmkv_kv_dequant_marked(const void* kv, const int32_t* block_table, int max_pages,
                                      const int32_t* seq_lens, int nseq, const uint64_t* mask, void* kvd,
                                      glmkv_stream_t stream) {
  if (nseq < 0 || max_pages < 0) return GLMKV_ERR_ARG;
  if (nseq == 0) return GLMKV_OK;
  if (!kv || !block_table || !seq_lens || !mask || !kvd) return GLMKV_ERR_ARG;
  if (!aligned(kv, 16) || !aligned(kvd, 16) || !aligned(mask, 8)) return GLMKV_ERR_ALIGN;
  const DeviceInfo* d = device_info();
  if (!d) return GLMKV_ERR_DEVICE;
  return launch(glm_kv_dequant_marked, d->sms * d->dq_ctas, DQ_THREADS, DQ_SMEM, stream, (const u8*)kv, block_table,
                max_pages, seq_lens, nseq, (const unsigned long long*)mask, (bf16*)kvd);
}

GLMKV_API int glmkv_topk_stream(int32_t* ind, const uint32_t* ks, const int32_t* klen, int32_t* tlen, int T,
                                glmkv_stream_t stream) {
  if (T < 0) return GLMKV_ERR_ARG;
  if (T == 0) return GLMKV_OK;
  if (!ind || !ks || !klen || !tlen) return GLMKV_ERR_ARG;
  if (!aligned(ind, 16)) return GLMKV_ERR_ALIGN;
  return launch(glm_topk_stream, T, TK_THREADS, 0, stream, ind, ks, klen, tlen, T);
}

GLMKV_API int glmkv_topk_slots(int32_t* ind, const int32_t* block_table, int max_pages, const int32_t* row_seq,
                               const int32_t* klen, int32_t* tlen, int T, glmkv_stream_t stream) {
  if (T < 0 || max_pages < 0) return GLMKV_ERR_ARG;
  if (T == 0) return GLMKV_OK;
  if (!ind || !block_table || !row_seq || !klen || !tlen) return GLMKV_ERR_ARG;
  if (!aligned(ind, 16)) return GLMKV_ERR_ALIGN;
  return launch(glm_topk_slots, T, TK_THREADS, 0, stream, ind, block_table, max_pages, row_seq, klen, tlen, T);
}

GLMKV_API int glmkv_q_post(const void* qb, int ldb, const void* rope, const int32_t* pos, void* qmla, void* iq,
                           const void* iw, float* wout, int full, int T, glmkv_stream_t stream) {
  if (T < 0) return GLMKV_ERR_ARG;
  if (T == 0) return GLMKV_OK;
  if (!qb || !rope || !pos || !qmla || (full && (!iq || !iw || !wout))) return GLMKV_ERR_ARG;
  if (ldb < HEADS * QHD + (full ? IH * ID : 0)) return GLMKV_ERR_ARG;
  if (ldb % 8 || !aligned(qb, 16) || !aligned(qmla, 16) || !aligned(rope, 8) ||
      (full && (!aligned(iq, 4) || !aligned(wout, 4) || !aligned(iw, 2))))
    return GLMKV_ERR_ALIGN;
  return launch(glm_q_post, (T + QP_WARPS - 1) / QP_WARPS, QP_THREADS, 0, stream, (const bf16*)qb, ldb,
                (const bf16*)rope, pos, (bf16*)qmla, (u8*)iq, (const bf16*)iw, wout, full, T);
}

GLMKV_API int glmkv_add_rms_quant(const void* a, void* res, const void* gamma, void* normed, void* q, void* sf,
                                  int sf_rows, int T, glmkv_stream_t stream) {
  if (T < 0) return GLMKV_ERR_ARG;
  if (T == 0) return GLMKV_OK;
  if (!res || !gamma || (q && (!sf || sf_rows < T))) return GLMKV_ERR_ARG;
  if (!aligned(res, 16) || (a && !aligned(a, 16)) || !aligned(gamma, 8) || (normed && !aligned(normed, 8)) ||
      (q && !aligned(q, 4)))
    return GLMKV_ERR_ALIGN;
  const DeviceInfo* d = device_info();
  if (!d) return GLMKV_ERR_DEVICE;
  return launch(glm_add_rms_quant, std::min(d->sms * d->arq_ctas, T), ARQ_THREADS, ARQ_SMEM, stream, (const bf16*)a,
                (bf16*)res, (const bf16*)gamma, (bf16*)normed, (u8*)q, (u8*)sf, sf_rows, T);
}

GLMKV_API int glmkv_quant(const void* x, int ldx, void* q, void* sf, int sf_rows, int K, int T, glmkv_stream_t stream) {
  if (T < 0 || K < 0) return GLMKV_ERR_ARG;
  if (T == 0 || K == 0) return GLMKV_OK;
  if (!x || !q || !sf || K % 128 || ldx < K || sf_rows < T) return GLMKV_ERR_ARG;
  if (ldx % 8 || !aligned(x, 16) || !aligned(q, 16) || !aligned(sf, 4)) return GLMKV_ERR_ALIGN;
  const long long warps = (long long)T * ((K / 128 + 3) / 4);
  const long long grid = (warps + QT_THREADS / 32 - 1) / (QT_THREADS / 32);
  if (grid > 0x7fffffffLL) return GLMKV_ERR_ARG;
  return launch(glm_quant, (int)grid, QT_THREADS, 0, stream, (const bf16*)x, ldx, (u8*)q, (u8*)sf, sf_rows, K, T);
}

GLMKV_API int glmkv_mqa_logits_paged(const void* iq, const void* idx, int n_pages, const int32_t* block_table,
                                     int max_pages, const int32_t* row_seq, const int32_t* klen, const float* w,
                                     float* logits, int stride, int R, glmkv_stream_t stream) {
  if (R < 0 || n_pages < 1 || max_pages < 1 || stride < 1) return GLMKV_ERR_ARG;
  if (R == 0) return GLMKV_OK;
  if (!iq || !idx || !block_table || !row_seq || !klen || !w || !logits) return GLMKV_ERR_ARG;
  if ((long long)R * IH > 0xffffffffll) return GLMKV_ERR_ARG;
  if (!aligned(iq, 16) || !aligned(idx, 16) || !aligned(w, 16) || !aligned(logits, 4)) return GLMKV_ERR_ALIGN;
  const DeviceInfo* d = device_info();
  if (!d) return GLMKV_ERR_DEVICE;
  const auto encode = tensor_map_encoder();
  if (!encode) return GLMKV_ERR_DEVICE;
  // iq as [R * 32 rows][128 B]; a box is one block of 8 rows (256 rows), 128-byte swizzle
  CUtensorMap tm_q, tm_k;
  const cuuint64_t q_dims[2] = {(cuuint64_t)ID, (cuuint64_t)R * IH}, q_strides[1] = {(cuuint64_t)ID};
  const cuuint32_t q_box[2] = {(cuuint32_t)ID, (cuuint32_t)MQ_N}, ones[3] = {1, 1, 1};
  if (encode(&tm_q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(iq), q_dims, q_strides, q_box, ones,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return GLMKV_ERR_ARG;
  // the indexer cache as [pages][64 rows][128 B], page stride 8448 B; a box is one page's keys
  const cuuint64_t k_dims[3] = {(cuuint64_t)ID, (cuuint64_t)PAGE, (cuuint64_t)n_pages};
  const cuuint64_t k_strides[2] = {(cuuint64_t)ID, (cuuint64_t)IDX_PAGE};
  const cuuint32_t k_box[3] = {(cuuint32_t)ID, (cuuint32_t)PAGE, 1};
  if (encode(&tm_k, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(idx), k_dims, k_strides, k_box, ones,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return GLMKV_ERR_ARG;
  const long long nch = ((stride + MQ_KEYS - 1) / MQ_KEYS + MQ_CHUNK - 1) / MQ_CHUNK;  // key chunks of a row block
  const int grid = (int)std::min<long long>(d->sms * d->mq_ctas, (long long)((R + MQ_ROWS - 1) / MQ_ROWS) * nch);
  return launch(glm_mqa_logits_paged, grid, MQ_THREADS, MQ_SMEM, stream, tm_q, tm_k, (const u8*)idx, n_pages,
                block_table, max_pages, row_seq, klen, w, logits, stride, R);
}

GLMKV_API int glmkv_launch_shape(const char* entry, int T, int* grid, int* block, int* smem_bytes) {
  if (!entry || !grid || !block || !smem_bytes || T < 0) return GLMKV_ERR_ARG;
  const auto is = [entry](const char* s) { return strcmp(entry, s) == 0; };
  if (is("glm_plan")) {
    *grid = (T + PLAN_THREADS - 1) / PLAN_THREADS, *block = PLAN_THREADS, *smem_bytes = 0;
  } else if (is("glm_quant")) {
    return GLMKV_ERR_ARG;  // its grid depends on K too: ceil(T * ceil(K / 512) / 8), block 256
  } else if (is("glm_add_rms_quant")) {
    const DeviceInfo* d = device_info();
    if (!d) return GLMKV_ERR_DEVICE;
    *grid = std::min(d->sms * d->arq_ctas, std::max(T, 1)), *block = ARQ_THREADS, *smem_bytes = ARQ_SMEM;
  } else if (is("glm_mqa_logits_paged")) {  // persistent: any grid works; one CTA an SM
    const DeviceInfo* d = device_info();
    if (!d) return GLMKV_ERR_DEVICE;
    *grid = d->sms * d->mq_ctas, *block = MQ_THREADS, *smem_bytes = MQ_SMEM;
  } else if (is("glm_q_post")) {
    *grid = (T + QP_WARPS - 1) / QP_WARPS, *block = QP_THREADS, *smem_bytes = 0;
  } else if (is("glm_topk_stream") || is("glm_topk_slots")) {
    *grid = T, *block = TK_THREADS, *smem_bytes = 0;
  } else if (is("glm_mark_rows") || is("glm_topk_stream_mark")) {
    const DeviceInfo* d = device_info();
    if (!d) return GLMKV_ERR_DEVICE;
    *grid = std::min(d->sms, std::max(1, (T + MK_RB - 1) / MK_RB)), *block = MK_THREADS, *smem_bytes = MK_SMEM;
  } else if (is("glm_kv_dequant") || is("glm_kv_dequant_marked") || is("glm_idx_gather") || is("glm_mla_prep") ||
             is("glm_mla_prep_fp8")) {
    const DeviceInfo* d = device_info();
    if (!d) return GLMKV_ERR_DEVICE;
    if (is("glm_kv_dequant") || is("glm_kv_dequant_marked")) {
      *grid = d->sms * d->dq_ctas, *block = DQ_THREADS, *smem_bytes = (int)DQ_SMEM;
    } else if (is("glm_idx_gather")) {
      *grid = d->sms * d->ga_ctas, *block = GA_THREADS, *smem_bytes = (int)GA_SMEM;
    } else {
      *grid = std::min(d->sms * d->prep_ctas, (T + PREP_WARPS - 1) / PREP_WARPS);
      *block = PREP_THREADS, *smem_bytes = PREP_SMEM;
    }
  } else {
    return GLMKV_ERR_ARG;
  }
  return GLMKV_OK;
}

GLMKV_API int glmkv_selftest_wait(uint64_t limit_ns, uint32_t* waited_ns, glmkv_stream_t stream) {
  if (!waited_ns || limit_ns == 0 || limit_ns > 1000000000ull) return GLMKV_ERR_ARG;
  glmkv_wait_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>((unsigned long long)limit_ns, waited_ns);
  return cudaGetLastError() == cudaSuccess ? GLMKV_OK : GLMKV_ERR_LAUNCH;
}

GLMKV_API int glmkv_fault_flags(uint32_t* flags, int clear) {
  if (!flags) return GLMKV_ERR_ARG;
  if (cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpyFromSymbol(flags, glmkv::g_fault, sizeof(uint32_t)) != cudaSuccess) {
    cudaGetLastError();
    return GLMKV_ERR_DEVICE;
  }
  if (clear) {
    const uint32_t zero = 0;
    if (cudaMemcpyToSymbol(glmkv::g_fault, &zero, sizeof zero) != cudaSuccess) {
      cudaGetLastError();
      return GLMKV_ERR_DEVICE;
    }
  }
  return GLMKV_OK;
}

GLMKV_API const char* glmkv_strerror(int code) {
  switch (code) {
    case GLMKV_OK: return "ok";
    case GLMKV_ERR_ARG: return "invalid argument (null pointer or size out of range)";
    case GLMKV_ERR_ALIGN: return "misaligned pointer or row stride";
    case GLMKV_ERR_DEVICE: return "no usable CUDA device";
    case GLMKV_ERR_LAUNCH: return "kernel launch (or the launcher's memset) failed";
    default: return "unknown glmkv error";
  }
}

GLMKV_API int glmkv_abi_version(void) { return 102; }
