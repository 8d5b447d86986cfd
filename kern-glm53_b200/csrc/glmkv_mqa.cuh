// The indexer's fp8 MQA logits read straight from the page-blocked indexer cache: the gather-free
// input format (the row after glm_idx_gather in kern-glm53's indexer, scripts/glm_ops.py:104-134).
//
//   logits[r * stride + p] = sum_h w[r, h] * relu( sum_d q[r, h, d] * k[p, d] ) * s[p]
//
// for every key position p < klen[r] of row r's sequence (row_seq[r]); q the e4m3 indexer query
// [R, 32, 128] (glm_q_post), w its head weights [R, 32] f32 (scale folded in), k / s the e4m3 key and
// f32 scale of position p: page block_table[seq][p / 64], row p % 64 of the indexer cache. This is
// the definition DeepGEMM's fp8_mqa_logits is tested against, in its compressed layout (row r's
// logits at [r][0, ke - ks)); the scale is non-negative, so relu(dot * s) = relu(dot) * s.
//
// One CTA per SM, warp-specialised, on Blackwell's tensor cores:
//  - warp 0: walks the work items (the warp reads a block's rows and block-table entries together)
//    and one lane issues bulk tensor copies (TMA, 128-byte swizzle) of a block of 8 query rows
//    (256 (row, head) rows of 128 bytes) and of key tiles (two 64-key pages, straight from the cache)
//    into a ring of shared-memory stages, each with a descriptor word for the MMA issuer;
//  - warp 1: allocates 512 TMEM columns; one lane, driven by the stage descriptors, issues
//    tcgen05.mma kind::f8f6f4 (e4m3 x e4m3 -> f32), M = 128 keys x N = 256 (row, head) x K = 128
//    (four K = 32 steps) into one of two TMEM accumulators, and commits each stage and accumulator
//    back to its barrier;
//  - warps 2..17: the epilogue, in two groups of 8 that take the tiles of even and odd index (the
//    two accumulators) so that their load and arithmetic phases interleave. Warp w reads TMEM lanes
//    32 (w % 4) .. + 31 (one key a thread) and the columns of four query rows, two at a time, then
//    relu, the head-weighted sum and the key's scale, and stores the logits (32 consecutive keys a
//    warp: 128-byte coalesced rows).
// A block of rows that spans two sequences is worked as two segments over the same query stage.
// Every wait is bounded; a wait that gives up sets the fault word, stops every role, waits for the
// copies and MMAs in flight and frees TMEM before returning.
#pragma once

#include <cuda.h>

#include <climits>

#include "glmkv_kernels.cuh"

namespace glmkv {

constexpr int MQ_ROWS = 8;                       // query rows a block: N = 8 x 32 heads
constexpr int MQ_N = MQ_ROWS * IH;               // 256 (row, head) rows
constexpr int MQ_KEYS = 2 * PAGE;                // keys a tile (M): two cache pages
constexpr int MQ_CHUNK = 16;                     // key tiles a work item (2048 keys)
constexpr int MQ_KSTAGES = 6;
constexpr int MQ_QBYTES = MQ_N * ID;             // 32,768 B: a query block, e4m3
constexpr int MQ_KBYTES = MQ_KEYS * ID;          // 16,384 B: a key tile, e4m3
constexpr int MQ_SCBYTES = MQ_KEYS * 4;          // 512 B: its keys' f32 scales
constexpr int MQ_EPI_WARPS = 16;                 // four a TMEM lane quarter, two query rows each
constexpr int MQ_THREADS = 32 * (2 + MQ_EPI_WARPS);
constexpr int MQ_TMEM_COLS = 2 * MQ_N;           // two f32 accumulators of 256 columns
constexpr int MQ_WBYTES = MQ_EPI_WARPS * 4 * IH * 4;  // each epilogue warp's four rows of head weights
constexpr int MQ_QTAB = 4096;                    // blocks whose largest klen is kept in shared memory
// A key stage's descriptor word, written by the producer before the stage's copies: the first tile
// of a work item (the MMA issuer then waits for the item's query stage), or the end of the launch.
constexpr uint32_t MQ_D_FIRST = 1u, MQ_D_END = 2u;
constexpr int MQ_SMEM = 1024 + 2 * MQ_QBYTES + MQ_KSTAGES * (MQ_KBYTES + MQ_SCBYTES) + MQ_WBYTES;  // + 1 KB: align
// instruction descriptor, kind::f8f6f4: D f32 (bits 4-5 = 1), A and B e4m3 (0), both K-major (0),
// N >> 3 at bits 17-22, M >> 4 at bits 24-28
constexpr uint32_t MQ_IDESC = (1u << 4) | ((uint32_t)(MQ_N >> 3) << 17) | ((uint32_t)(MQ_KEYS >> 4) << 24);

// Shared-memory matrix descriptor of a K-major operand in the 128-byte swizzle layout: rows of 128
// bytes, 8-row groups 1024 bytes apart (SBO), the tile 1024-byte aligned (base offset 0). Start
// address bits 0-13 (>> 4), LBO bits 16-29 (unused for this layout: 16 B), SBO bits 32-45, version 1
// at bits 46-47, layout 2 (128-byte swizzle) at bits 61-63. A K step of 32 bytes adds 2 to the start.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The barrier's phase completes once every tcgen05 operation this thread issued before has.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// 16 f32 columns of this warp's 32 TMEM lanes (one lane a thread) at `taddr`. The registers are valid
// after tc_ld16_wait; every register of a load issued before that wait passes through it (or through
// tc_ld16_after), so that no read of them moves above the wait.
__device__ __forceinline__ void tc_ld16_issue(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tc_ld16_wait(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]),
        "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
      :: "memory");
}
__device__ __forceinline__ void tc_ld16_after(uint32_t (&r)[16]) {
  asm volatile(""
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]),
        "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
      :: "memory");
}
// try_wait with a suspend-time hint: the warp sleeps until the phase completes (or `hint_ns` pass)
// instead of spinning, so waiting warps leave the issue slots to the working ones.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// A bounded wait that also gives up as soon as another role has (the CTA's abort word is set).
__device__ __forceinline__ bool mq_wait(uint32_t bar, uint32_t parity, const volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait_sleep(bar, parity, 20000u)) {
    if (*abort) return false;
    if (global_ns() - t0 > WAIT_LIMIT_NS) return false;
  }
  return true;
}

// The work of a launch is a grid of items (query block qb of 8 rows, key chunk c of 16 tiles = 2048
// positions), numbered chunk-major: item i = c * nqb + qb, so the first chunk of every block comes
// before any second chunk. Item i goes to CTA i % G. An item covers, in each segment of its block (a
// run of rows of one sequence), the key tiles c * 16 .. c * 16 + 15 below the segment's largest klen;
// an item with none is skipped by every role alike, and every role walks the items in the same order.
// MqItems steps through this CTA's items, blockIdx.x, + G, + 2 G, ..., as (block qb, chunk c) without
// a division a step: G = cg * nqb + qg. The walk ends at the first chunk no row of the launch reaches.
struct MqItems {
  int qb, c, nqb, nch, qg, cg;
  __device__ __forceinline__ MqItems(int nqb_, int nch_)
      : qb((int)(blockIdx.x % nqb_)), c((int)(blockIdx.x / nqb_)), nqb(nqb_), nch(nch_),
        qg((int)(gridDim.x % nqb_)), cg((int)(gridDim.x / nqb_)) {}
  __device__ __forceinline__ bool valid() const { return c < nch; }
  __device__ __forceinline__ void next() {
    qb += qg;
    c += cg;
    if (qb >= nqb) qb -= nqb, ++c;
  }
};
// relu(x) * 2^-25 on the FMA pipe: saturate(x * 2^-25 + 0), which clamps to [0, 1]. A dot product of
// 128 e4m3 pairs is below 128 * 448^2 < 2^25 in magnitude, so this is relu(x) scaled by an exact
// power of two (the smallest nonzero |x|, 2^-18, stays a normal number), and with the head weights
// scaled by 2^25 each product w * relu(x) rounds exactly as before. A NaN gives 0, as fmaxf(NaN, 0).
__device__ __forceinline__ float relu_s(float x) {
  float d;
  asm("fma.rn.sat.f32 %0, %1, 0f33000000, 0f00000000;" : "=f"(d) : "f"(x));
  return d;
}
struct MqSegment {
  int sb, se, seq, kmax, kb0, kb1;  // rows [sb, se), key tiles [kb0, kb1)
};
// The rows of block qb as a warp holds them: lane j < 8 has row qb * 8 + j's sequence and klen
// (-1 and 0 past R): two loads a lane, one round trip for the block.
struct MqRows {
  int seq, kl;
};
__device__ __forceinline__ MqRows mq_load_rows(const int* __restrict__ row_seq, const int* __restrict__ klen, int R,
                                               int qb) {
  const int l = threadIdx.x & 31, r = qb * MQ_ROWS + l;
  MqRows v{-1, 0};
  if (l < MQ_ROWS && r < R) v = MqRows{__ldg(row_seq + r), __ldg(klen + r)};
  return v;
}
// f(segment) for each segment (a run of rows of one sequence) of block qb with key tiles in chunk c;
// false as soon as f returns false. Warp-collective: every lane calls it with the block's rows.
template <class F>
__device__ __forceinline__ bool mq_segments(const MqRows& v, int R, int qb, int c, F&& f) {
  const int l = threadIdx.x & 31, r0 = qb * MQ_ROWS, n = min(MQ_ROWS, R - r0);
  const int prev = __shfl_up_sync(FULL, v.seq, 1);
  unsigned starts = __ballot_sync(FULL, l < n && (l == 0 || v.seq != prev));  // the first row of each segment
  while (starts) {
    const int sb = __ffs(starts) - 1;
    starts &= starts - 1;
    const int se = starts ? __ffs(starts) - 1 : n;
    const int kmax = __reduce_max_sync(FULL, l >= sb && l < se ? v.kl : INT_MIN);
    const int s = __shfl_sync(FULL, v.seq, sb);
    const int nkb = (kmax + MQ_KEYS - 1) / MQ_KEYS;
    const int kb0 = c * MQ_CHUNK, kb1 = min(kb0 + MQ_CHUNK, nkb);
    if (kb0 < kb1 && !f(MqSegment{r0 + sb, r0 + se, s, kmax, kb0, kb1})) return false;
  }
  return true;
}
// Whether item (qb, c) has any tile: a segment has tiles in chunk c when its largest klen passes
// c * 2048, so the item has some when the block's largest klen does. `qmax` holds every block's
// largest klen when the launch has at most MQ_QTAB blocks; otherwise the warp reads the rows here.
__device__ __forceinline__ bool mq_item_has_tiles(const int* qmax, const int* __restrict__ klen, int R, int nqb, int qb,
                                                  int c) {
  int m;
  if (nqb <= MQ_QTAB) {
    m = qmax[qb];
  } else {
    const int l = threadIdx.x & 31, r = qb * MQ_ROWS + l;
    m = __reduce_max_sync(FULL, l < MQ_ROWS && r < R ? max(__ldg(klen + r), 0) : 0);
  }
  return m > c * MQ_CHUNK * MQ_KEYS;
}
// Moves `it` to the first item at or after it with key tiles. Warp-collective.
__device__ __forceinline__ void mq_skip_empty(MqItems& it, const int* qmax, const int* __restrict__ klen, int R) {
  while (it.valid() && !mq_item_has_tiles(qmax, klen, R, it.nqb, it.qb, it.c)) it.next();
}

__device__ __forceinline__ void mq_logits(const CUtensorMap* tm_q, const CUtensorMap* tm_k, const u8* __restrict__ idx,
                                          int n_pages, const int* __restrict__ block_table, int max_pages,
                                          const int* __restrict__ row_seq, const int* __restrict__ klen,
                                          const float* __restrict__ w, float* __restrict__ logits, int stride, int R) {
  extern __shared__ __align__(1024) u8 mq_smem_raw[];
  __shared__ __align__(8) unsigned long long q_full[2], q_empty[2], k_full[MQ_KSTAGES], k_empty[MQ_KSTAGES],
      acc_full[2], acc_empty[2], mma_done;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  __shared__ uint32_t kdesc[MQ_KSTAGES];  // each key stage's descriptor word (MQ_D_*)
  __shared__ unsigned kmax_all;  // the largest klen of the launch's rows
  __shared__ int qmax[MQ_QTAB];  // each block's largest klen (launches of at most MQ_QTAB blocks)
  const int tid = threadIdx.x, warp = tid >> 5, l = tid & 31;
  const uint32_t sbase = (smem_u32(mq_smem_raw) + 1023u) & ~1023u;  // 1024-aligned for the swizzle
  const uint32_t qbuf = sbase, kbuf = sbase + 2 * MQ_QBYTES, scbuf = kbuf + MQ_KSTAGES * MQ_KBYTES;
  const uint32_t wbuf = scbuf + MQ_KSTAGES * MQ_SCBYTES;
  u8* const sgen = mq_smem_raw + (sbase - smem_u32(mq_smem_raw));  // generic pointer of sbase
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&q_full[i]), 1);
      mbar_init(smem_u32(&q_empty[i]), 1);
      mbar_init(smem_u32(&acc_full[i]), 1);
      mbar_init(smem_u32(&acc_empty[i]), MQ_EPI_WARPS / 2);  // the group of that parity
    }
    for (int i = 0; i < MQ_KSTAGES; ++i) {
      mbar_init(smem_u32(&k_full[i]), 1);
      mbar_init(smem_u32(&k_empty[i]), 1 + MQ_EPI_WARPS / 2);  // the MMAs, and the group's warps once they hold the scales
    }
    mbar_init(smem_u32(&mma_done), 1);
    mbar_init_fence();
    abort_flag = 0;
    kmax_all = 0;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(MQ_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  pdl_trigger();  // one CTA per SM, all resident
  pdl_wait();
  const volatile int* abort = &abort_flag;
  auto give_up = [&]() {
    atomicOr(&g_fault, FAULT_WAIT_TIMEOUT);
    abort_flag = 1;
  };
  const int nqb = (R + MQ_ROWS - 1) / MQ_ROWS;
  {  // every block's largest klen, and the launch's: the chunks any row needs (stride bounds the stores)
    unsigned m = 0;
    if (nqb <= MQ_QTAB) {
      // one row a thread (rows of a block in 8 consecutive lanes), the block's max over those lanes
      for (int r0 = 0; r0 < R; r0 += MQ_THREADS) {
        const int r = r0 + tid;
        unsigned k = r < R ? (unsigned)max(klen[r], 0) : 0u;
        k = max(k, __shfl_xor_sync(FULL, k, 1));
        k = max(k, __shfl_xor_sync(FULL, k, 2));
        k = max(k, __shfl_xor_sync(FULL, k, 4));
        if ((r & 7) == 0 && r < R) qmax[r >> 3] = (int)k;
        m = max(m, k);
      }
    } else {
      for (int r = tid; r < R; r += MQ_THREADS) m = max(m, (unsigned)max(klen[r], 0));
    }
    m = __reduce_max_sync(FULL, m);
    if (l == 0) atomicMax(&kmax_all, m);
  }
  __syncthreads();
  const unsigned kcap = min(kmax_all, (unsigned)stride);
  const int nch = (int)(((kcap + MQ_KEYS - 1) / MQ_KEYS + MQ_CHUNK - 1) / MQ_CHUNK);

  if (warp == 0) {
    // ---------------------------------------------------------------- producer: bulk tensor copies
    uint32_t kit = 0, qit = 0, k_issued = 0;
    int q_issued = 0;
    bool ok = true;
    MqItems it(nqb, nch);
    mq_skip_empty(it, qmax, klen, R);
    while (ok && it.valid()) {
      const int qb = it.qb, c = it.c;
      const MqRows rows = mq_load_rows(row_seq, klen, R, qb);
      const int qs = qit & 1;
      if (l == 0) {
        ok = mq_wait(smem_u32(&q_empty[qs]), ((qit >> 1) & 1) ^ 1, abort);
        if (ok) {
          mbar_arrive_expect_tx(smem_u32(&q_full[qs]), MQ_QBYTES);
          tma_load_2d(qbuf + qs * MQ_QBYTES, tm_q, 0, qb * MQ_ROWS * IH, smem_u32(&q_full[qs]));
        }
      }
      ok = __shfl_sync(FULL, ok, 0);
      if (!ok) break;
      q_issued |= 1 << qs;
      ++qit;
      uint32_t first = MQ_D_FIRST;
      ok = mq_segments(rows, R, qb, c, [&](const MqSegment& g) {
        // lane j holds the page of position block 2 kb0 + j (the item's up to 32 pages)
        const int pj = 2 * g.kb0 + l;
        int pg = -1;
        if (pj * PAGE < g.kmax) {  // a position the rows need: its page must be in the table and the pool
          if (pj < max_pages) {
            pg = block_table[(size_t)g.seq * max_pages + pj];
            if (pg >= n_pages) pg = -1;
          }
          if (pg < 0) atomicOr(&g_fault, FAULT_BAD_PAGE);
        }
        for (int kb = g.kb0; kb < g.kb1; ++kb) {
          const int st = kit % MQ_KSTAGES;
          const int p0 = __shfl_sync(FULL, pg, 2 * (kb - g.kb0)), p1 = __shfl_sync(FULL, pg, 2 * (kb - g.kb0) + 1);
          bool okk = true;
          if (l == 0) {
            okk = mq_wait(smem_u32(&k_empty[st]), ((kit / MQ_KSTAGES) & 1) ^ 1, abort);
            if (okk) {
              kdesc[st] = first;  // published by the arrive below
              const uint32_t bytes = (p0 >= 0 ? MQ_KBYTES / 2 + MQ_SCBYTES / 2 : 0) +
                                     (p1 >= 0 ? MQ_KBYTES / 2 + MQ_SCBYTES / 2 : 0);
              mbar_arrive_expect_tx(smem_u32(&k_full[st]), bytes);
              const int pp[2] = {p0, p1};
#pragma unroll
              for (int j = 0; j < 2; ++j)
                if (pp[j] >= 0) {
                  tma_load_3d(kbuf + st * MQ_KBYTES + j * (MQ_KBYTES / 2), tm_k, 0, 0, pp[j], smem_u32(&k_full[st]));
                  tma_load_1d(scbuf + st * MQ_SCBYTES + j * (MQ_SCBYTES / 2),
                              idx + (size_t)pp[j] * IDX_PAGE + PAGE * ID, MQ_SCBYTES / 2, smem_u32(&k_full[st]));
                }
            }
          }
          if (!__shfl_sync(FULL, okk, 0)) return false;
          k_issued |= 1u << st;
          first = 0;
          ++kit;
        }
        return true;
      });
      it.next();
      mq_skip_empty(it, qmax, klen, R);
    }
    if (ok && l == 0) {  // the end marker: a stage with no copies, completed by a plain arrive
      const int st = kit % MQ_KSTAGES;
      ok = mq_wait(smem_u32(&k_empty[st]), ((kit / MQ_KSTAGES) & 1) ^ 1, abort);
      if (ok) {
        kdesc[st] = MQ_D_END;
        mbar_arrive(smem_u32(&k_full[st]));
        k_issued |= 1u << st;
        ++kit;
      }
    }
    if (!ok && l == 0) give_up();
    if (l == 0) {  // wait (bounded) for every copy still in flight: the last phase of each stage used
      for (int st = 0; st < MQ_KSTAGES; ++st)
        if (k_issued & (1u << st)) {
          const uint32_t last = (kit - 1 - ((kit - 1 - st) % MQ_KSTAGES)) / MQ_KSTAGES;  // index of its last use
          mbar_wait_bounded(smem_u32(&k_full[st]), last & 1, WAIT_LIMIT_NS);
        }
      for (int qs = 0; qs < 2; ++qs)
        if (q_issued & (1 << qs)) {
          const uint32_t last = (qit - 1 - ((qit - 1 - qs) & 1)) >> 1;  // index of its last use
          mbar_wait_bounded(smem_u32(&q_full[qs]), last & 1, WAIT_LIMIT_NS);
        }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issue (one lane)
    // Driven by the stage descriptors: no walk of the items here, so the lane does little besides
    // waiting and issuing. A work item's query stage is released when the next item starts.
    if (l == 0) {
      uint32_t st = 0, kph = 0, tile = 0, qit = 0;
      bool ok = true, issued = false;
      uint64_t bdesc = 0;
      for (;;) {
        if (!(ok = mq_wait(smem_u32(&k_full[st]), kph, abort))) break;
        const uint32_t d = kdesc[st];
        if (d & MQ_D_END) break;
        if (d & MQ_D_FIRST) {
          if (qit > 0) tc_commit(smem_u32(&q_empty[(qit - 1) & 1]));
          if (!(ok = mq_wait(smem_u32(&q_full[qit & 1]), (qit >> 1) & 1, abort))) break;
          bdesc = sw128_desc(qbuf + (qit & 1) * MQ_QBYTES);
          ++qit;
        }
        const uint32_t a = tile & 1;
        if (!(ok = mq_wait(smem_u32(&acc_empty[a]), ((tile >> 1) & 1) ^ 1, abort))) break;
        tc_fence_after();
        const uint64_t adesc = sw128_desc(kbuf + st * MQ_KBYTES);
#pragma unroll
        for (int kk = 0; kk < ID / 32; ++kk)
          tc_mma(tmem + a * MQ_N, adesc + 2 * kk, bdesc + 2 * kk, MQ_IDESC, kk > 0);
        issued = true;
        tc_commit(smem_u32(&k_empty[st]));
        tc_commit(smem_u32(&acc_full[a]));
        ++tile;
        if (++st == MQ_KSTAGES) st = 0, kph ^= 1;
      }
      if (!ok) give_up();
      if (issued) {  // every MMA has completed before TMEM is freed
        tc_commit(smem_u32(&mma_done));
        mbar_wait_bounded(smem_u32(&mma_done), 0, WAIT_LIMIT_NS);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue: TMEM -> logits
    // Two groups of 8 warps: group gp works the tiles of parity gp (accumulator gp), so the groups'
    // load and arithmetic phases interleave. Warp e of a group: TMEM lane quarter warp % 4, query rows
    // 4 cq .. 4 cq + 3 of a block (two pairs).
    const int e = warp - 2, gp = e >> 3;
    const int qd = warp & 3, cq = (e & 7) >> 2;
    float* wsm = reinterpret_cast<float*>(sgen + (wbuf - sbase)) + e * 4 * IH;
    uint32_t est = 0, tpar = 0, eph = 0;  // key stage and parity of the next tile; the group accumulator's phase
    bool ok = true;
    MqItems it(nqb, nch);
    mq_skip_empty(it, qmax, klen, R);
    while (ok && it.valid()) {
      const int qb = it.qb, c = it.c;
      const MqRows rows = mq_load_rows(row_seq, klen, R, qb);
      const int r4 = qb * MQ_ROWS + 4 * cq;  // this warp's rows r4 .. r4 + 3
      {  // head weights (zero past R) x 2^25, pair j interleaved by head: wsm[64 j + 2 h + i] = w[r4 + 2 j + i][h]
        const int rr = l >> 3, h4 = 4 * (l & 7);
        const float4 v = r4 + rr < R ? __ldg(reinterpret_cast<const float4*>(w + (size_t)(r4 + rr) * IH + h4))
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
        float* d = wsm + 64 * (rr >> 1) + (rr & 1);
        __syncwarp();
        d[2 * h4] = v.x * 33554432.f;  // w * 2^25 (exact): relu(x) * w = relu_s(x) * (w * 2^25)
        d[2 * h4 + 2] = v.y * 33554432.f;
        d[2 * h4 + 4] = v.z * 33554432.f;
        d[2 * h4 + 6] = v.w * 33554432.f;
        __syncwarp();
      }
      int klr[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) klr[i] = __shfl_sync(FULL, rows.kl, 4 * cq + i);
      float* const out0 = logits + (size_t)r4 * stride;
      ok = mq_segments(rows, R, qb, c, [&](const MqSegment& g) {
        // the positions each row stores: below its klen and the stride, in its own segment only
        int lim[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) lim[i] = r4 + i >= g.sb && r4 + i < g.se ? min(klr[i], stride) : 0;
        const int limp0 = max(lim[0], lim[1]), limp1 = max(lim[2], lim[3]);
        for (int kb = g.kb0; kb < g.kb1; ++kb) {
          const uint32_t st = est;
          const bool mine = tpar == (uint32_t)gp;
          if (++est == MQ_KSTAGES) est = 0;
          tpar ^= 1;
          if (!mine) continue;  // the other group's tile
          const bool okw = mq_wait(smem_u32(&acc_full[gp]), eph, abort);
          if (__any_sync(FULL, !okw)) return false;  // the warp leaves together: tcgen05.ld is warp-collective
          tc_fence_after();
          // the key's scale into a register, and the stage back to the producer: the MMAs have read
          // its keys (they completed before acc_full), so the next copies need not wait for the sums
          const float scale = reinterpret_cast<const float*>(sgen + (scbuf - sbase) + st * MQ_SCBYTES)[32 * qd + l];
          __syncwarp();
          if (l == 0) mbar_arrive(smem_u32(&k_empty[st]));
          const int p = kb * MQ_KEYS + 32 * qd + l;  // this thread's key position
          const int p0 = kb * MQ_KEYS + 32 * qd;
          if (p0 < max(limp0, limp1)) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              if (p0 >= (j ? limp1 : limp0)) continue;
              // sum over heads of w * relu(v) for both rows of the pair: two chains of packed FMAs (even
              // and odd heads), each lane holding (row 2 j, row 2 j + 1); heads 0 .. 15, then 16 .. 31
              const uint32_t t0 = tmem + gp * MQ_N + ((uint32_t)(32 * qd) << 16) + (4 * cq + 2 * j) * IH;
              const float* wp = wsm + 64 * j;
              float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
              uint32_t ua[16], ub[16], va[16], vb[16];
              tc_ld16_issue(t0, ua);
              tc_ld16_issue(t0 + IH, ub);
              tc_ld16_wait(ua);
              tc_ld16_after(ub);
              tc_ld16_issue(t0 + 16, va);  // the second half is on its way while the first is summed
              tc_ld16_issue(t0 + IH + 16, vb);
#pragma unroll
              for (int h = 0; h < 16; h += 2) {
                const float4 ww = *reinterpret_cast<const float4*>(wp + 2 * h);
                acc0 = fma2(make_float2(ww.x, ww.y),
                            make_float2(relu_s(__uint_as_float(ua[h])), relu_s(__uint_as_float(ub[h]))), acc0);
                acc1 = fma2(make_float2(ww.z, ww.w),
                            make_float2(relu_s(__uint_as_float(ua[h + 1])), relu_s(__uint_as_float(ub[h + 1]))), acc1);
              }
              tc_ld16_wait(va);
              tc_ld16_after(vb);
#pragma unroll
              for (int h = 0; h < 16; h += 2) {
                const float4 ww = *reinterpret_cast<const float4*>(wp + 2 * (16 + h));
                acc0 = fma2(make_float2(ww.x, ww.y),
                            make_float2(relu_s(__uint_as_float(va[h])), relu_s(__uint_as_float(vb[h]))), acc0);
                acc1 = fma2(make_float2(ww.z, ww.w),
                            make_float2(relu_s(__uint_as_float(va[h + 1])), relu_s(__uint_as_float(vb[h + 1]))), acc1);
              }
              const float2 sum = make_float2(__fadd_rn(acc0.x, acc1.x), __fadd_rn(acc0.y, acc1.y));
              // streaming stores: the logits pass through L2 without evicting the keys the other row
              // blocks of the sequence still read
              float* const o = out0 + (size_t)(2 * j) * stride;
              if (p < lim[2 * j]) __stcs(o + p, __fmul_rn(sum.x, scale));
              if (p < lim[2 * j + 1]) __stcs(o + stride + p, __fmul_rn(sum.y, scale));
            }
          }
          tc_fence_before();
          __syncwarp();
          if (l == 0) mbar_arrive(smem_u32(&acc_empty[gp]));  // the accumulator is read
          eph ^= 1;
        }
        return true;
      });
      it.next();
      mq_skip_empty(it, qmax, klen, R);
    }
    if (!ok && l == 0) give_up();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(MQ_TMEM_COLS) : "memory");
  }
}

}  // namespace glmkv

// The indexer's MQA logits of rows 0 .. R - 1 over their sequences' keys, read from the indexer
// cache pages (no gather). tm_q maps iq as [R * 32 rows][128 B] (box 256 rows, 128-byte swizzle);
// tm_k maps the indexer cache as [pages][64 rows][128 B] with strides 8448 and 128 B (box one page,
// 128-byte swizzle). idx is the same cache of n_pages pages (the key scales at each page's tail);
// a block-table entry outside 0 .. n_pages - 1, or a key position past the table's max_pages pages,
// is skipped and flagged (the logits of its keys are then not defined). No counterpart
// among the glue kernels: it replaces the gather plus DeepGEMM's MQA logits.
//   persistent: grid = SMs, block 576, dynamic smem MQ_SMEM (176,128 B)
extern "C" __global__ void __launch_bounds__(glmkv::MQ_THREADS, 1)
    glm_mqa_logits_paged(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const glmkv::u8* __restrict__ idx, int n_pages, const int* __restrict__ block_table,
                         int max_pages,
                         const int* __restrict__ row_seq, const int* __restrict__ klen, const float* __restrict__ w,
                         float* __restrict__ logits, int stride, int R) {
  glmkv::mq_logits(&tm_q, &tm_k, idx, n_pages, block_table, max_pages, row_seq, klen, w, logits, stride, R);
}
