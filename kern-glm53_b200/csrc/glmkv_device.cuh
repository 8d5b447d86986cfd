// Device-side building blocks of the KV-cache path: the cache geometry, the exact conversions the
// reference arithmetic is defined by, warp reductions that reproduce the reference's association
// order, and the mbarrier / bulk-copy (TMA) primitives of the page pipelines.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace glmkv {

typedef __nv_bfloat16 bf16;
typedef unsigned char u8;

// Geometry of GLM-5.3's latent and indexer caches (kern-glm53 source/glm_glue.cu:26-40,
// scripts/gen.py:51-61).
constexpr int QL = 2048;                   // q_a width
constexpr int KVL = 512;                   // kv_norm width
constexpr int HALF = 32;                   // rope pairs
constexpr int MLA = KVL + 2 * HALF;        // 576 values in a bf16 latent row
constexpr int ID = 128;                    // indexer key width
constexpr int TOPK = 2048;                 // indexer picks a row
constexpr int PAGE = 64;                   // tokens a cache page
constexpr int IDX_PAGE = PAGE * (ID + 4);  // 8448 B: 64 e4m3 keys, then their 64 f32 scales
constexpr int KV8 = KVL + 16 + 2 * 64;     // 656 B: fp8_ds_mla row (512 e4m3 | 4 f32 | 64 bf16)
constexpr int KVB = MLA * 2;               // 1152 B: bf16 latent row
constexpr int KV8_PAGE = PAGE * KV8;       // 41984 B
constexpr float EPS = 1e-5f;

constexpr unsigned FULL = 0xffffffffu;

// Fault word of the module: bits set by kernels that hit a bounded wait's limit or an invalid page.
// The host reads and clears it through glmkv_fault_flags().
enum : unsigned { FAULT_WAIT_TIMEOUT = 1u, FAULT_BAD_PAGE = 2u, FAULT_BAD_PICK = 4u };

// ------------------------------------------------------------------------------------------ loads

__device__ __forceinline__ uint2 ld_stream_v2(const void* p) {
  uint2 v;
  asm("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ld_stream_u32(const void* p) {
  uint32_t v;
  asm("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ld_stream_v4u(const void* p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ int4 ld_stream_v4(const void* p) {
  int4 v;
  asm("ld.global.nc.L1::no_allocate.v4.s32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ void st_stream_v4(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// ------------------------------------------------------------------------------------------ formats

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// bf16 round to nearest even and back (kern-glm53 glm_glue.cu:43 `rnd`).
__device__ __forceinline__ float rnd(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Four values to e4m3 with satfinite, first value in the low byte (glm_glue.cu:76-79).
__device__ __forceinline__ uint32_t fp8x4(float a, float b, float c, float d) {
  const __nv_fp8x4_e4m3 q(make_float4(a, b, c, d));
  return *reinterpret_cast<const uint32_t*>(&q);
}
__device__ __forceinline__ uint16_t fp8x2(float a, float b) {
  return __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
}

// The UE8M0 scale of a block (glm_glue.cu:68-74): the exponent byte of the correctly rounded
// q = max(amax, eps) / 448, plus one when q is not a power of two; the scale is that power of two.
// Computed on the bits of x = max(amax, eps) without the division. With x = 2^e (1 + M / 2^23),
// x / 448 = 2^(e - 9) (1 + M / 2^23) * 8 / 7, and (1 + M / 2^23) * 8 / 7 lies in [8/7, 2) for
// M <= 0x600000 (exactly 2 at M = 0x600000, q = 2^(e - 8)) and in (2, 16/7) above it. The nearest
// f32 to q never crosses those powers of two, because a quotient within half an ulp of one would need
// x within 2^-24 of 7 * 2^k, and the only f32 there is 7 * 2^k itself. So the byte is
// E - 8 + (M > 0x600000), E the biased exponent of x. x is a normal number (x >= eps >= 1e-10);
// x = inf gives 255 as the quotient would. eps keeps NaN out (fmaxf drops it).
__device__ __forceinline__ unsigned ue8m0_byte(float amax, float eps) {
  const unsigned b = __float_as_uint(fmaxf(amax, eps));
  const unsigned E = b >> 23, M = b & 0x7fffffu;
  return E == 255u ? 255u : E - 8u + (M > 0x600000u ? 1u : 0u);
}
__device__ __forceinline__ float ue8m0(float amax, float eps, unsigned* e) {
  *e = ue8m0_byte(amax, eps);
  return __uint_as_float(*e << 23);
}
// The same byte through the division itself (the reference's form); identical results. The append's
// q quant uses this one: measured faster there, where the division overlaps the reductions.
__device__ __forceinline__ float ue8m0_div(float amax, float eps, unsigned* e) {
  const unsigned b = __float_as_uint(__fdiv_rn(fmaxf(amax, eps), 448.f));
  *e = ((b >> 23) & 0xffu) + ((b & 0x7fffffu) != 0 ? 1u : 0u);
  return __uint_as_float(*e << 23);
}
// 1 / 2^(e - 127) exactly (the reciprocal of a UE8M0 scale): v * this rounds exactly as v / scale.
__device__ __forceinline__ float ue8m0_inv(unsigned e) {
  return e <= 253u ? __uint_as_float((254u - e) << 23) : (e == 254u ? __uint_as_float(0x00400000u) : 0.f);
}

// Two e4m3 bytes -> two bf16 of (value * sc): the f32 product rounded, then rounded to bf16
// (glm_glue.cu:405-408). e4m3 -> f16 -> f32 is exact.
__device__ __forceinline__ uint32_t dequant2(uint16_t pair, float sc) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(pair, __NV_E4M3);
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
  return pack_bf16x2(__fmul_rn(f.x, sc), __fmul_rn(f.y, sc));
}

// ------------------------------------------------------------------------------------------ reductions

// `warp_sum` / `warp_max` of the reference (glm_glue.cu:45-54): xor butterfly, offsets 16 .. 1.
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
  return v;
}

// The reference's 256-thread `block_sum` (glm_glue.cu:57-65) evaluated by ONE warp that holds, in
// v[w], the partial of thread (warp w, lane l) for all eight virtual warps w. Each butterfly level
// adds the same two operands as the reference's `v += shfl_xor(v, o)` of virtual warp w (a
// reduce-scatter: half the values travel at each of the first three levels), so every sum is
// bitwise the reference's. After five levels lane l holds warp total S_w, w = (l >> 2) & 7. The
// block stage then combines warp totals in the reference's order: w ^ 4, w ^ 2, w ^ 1 (its levels
// 16 and 8 add exact zeros). Every lane returns the block total.
__device__ __forceinline__ float block_sum8(const float (&v)[8], int l) {
  const bool b4 = l & 16, b3 = l & 8, b2 = l & 4;
  float a[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float send = b4 ? v[k] : v[k + 4], keep = b4 ? v[k + 4] : v[k];
    a[k] = keep + __shfl_xor_sync(FULL, send, 16);
  }
  float b[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const float send = b3 ? a[k] : a[k + 2], keep = b3 ? a[k + 2] : a[k];
    b[k] = keep + __shfl_xor_sync(FULL, send, 8);
  }
  float c;
  {
    const float send = b2 ? b[0] : b[1], keep = b2 ? b[1] : b[0];
    c = keep + __shfl_xor_sync(FULL, send, 4);
  }
  c += __shfl_xor_sync(FULL, c, 2);
  c += __shfl_xor_sync(FULL, c, 1);
  c += __shfl_xor_sync(FULL, c, 16);
  c += __shfl_xor_sync(FULL, c, 8);
  c += __shfl_xor_sync(FULL, c, 4);
  return c;
}

// Max over the warp of eight per-lane values v[w], scattered: lane l returns the max of v[w] for
// w = (l >> 2) & 7. Max is exact, so only the lane layout matters.
__device__ __forceinline__ float max8_scatter(const float (&v)[8], int l) {
  const bool b4 = l & 16, b3 = l & 8, b2 = l & 4;
  float a[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float send = b4 ? v[k] : v[k + 4], keep = b4 ? v[k + 4] : v[k];
    a[k] = fmaxf(keep, __shfl_xor_sync(FULL, send, 16));
  }
  float b[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const float send = b3 ? a[k] : a[k + 2], keep = b3 ? a[k + 2] : a[k];
    b[k] = fmaxf(keep, __shfl_xor_sync(FULL, send, 8));
  }
  const float send = b2 ? b[0] : b[1], keep = b2 ? b[1] : b[0];
  float c = fmaxf(keep, __shfl_xor_sync(FULL, send, 4));
  c = fmaxf(c, __shfl_xor_sync(FULL, c, 2));
  return fmaxf(c, __shfl_xor_sync(FULL, c, 1));
}

// ------------------------------------------------------------------------------------------ mbarrier + TMA

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Wait for the barrier phase with the given parity, giving up after `limit_ns` nanoseconds.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - t0 > limit_ns) return false;
  return true;
}
// One bulk (TMA) copy of `bytes` (a multiple of 16, both addresses 16-byte aligned) from global
// memory of THIS GPU into this CTA's shared memory, completing on the mbarrier.
__device__ __forceinline__ void tma_load_1d(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
// A bulk prefetch of `bytes` (a multiple of 16, the address 16-byte aligned) of THIS GPU's global memory
// into L2. A hint: it moves no data into the program's view and changes no value.
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Programmatic dependent launch. A kernel launched with programmatic stream serialization may start
// while the kernel before it on the stream is finishing; it must not touch global memory before
// pdl_wait(), which returns once that kernel has completed and its writes are visible (at once when
// the launch had no programmatic dependency). pdl_trigger() lets the next kernel start early; it is
// issued only when every CTA of this grid is already resident, so early dependents never hold
// resources that this grid's own CTAs still need.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// The pages of every sequence in order (kern-glm53 glm_glue.cu:360-371, 385-395): page j of
// sequence s covers its rows [64 j, min(64 j + 64, len)) and lands at stream rows goff(s) + 64 j,
// goff(s) being the 32-bit unsigned sum of the lengths before s. A cursor walks them forward, so a
// CTA that visits increasing global page numbers pays O(nseq + pages) in total.
struct PageCursor {
  const int* seq_lens;
  int nseq, s, len, npages;
  long long first;  // global number of sequence s's first page
  unsigned goff;

  __device__ __forceinline__ void init(const int* sl, int n) {
    seq_lens = sl;
    nseq = n;
    s = 0;
    first = 0;
    goff = 0;
    fetch();
  }
  __device__ __forceinline__ void fetch() {
    if (s < nseq) {
      len = seq_lens[s];
      npages = (len + PAGE - 1) / PAGE;
    }
  }
  // Move to global page g (never backwards); false once g is past the last page.
  __device__ __forceinline__ bool seek(long long g) {
    while (s < nseq && g >= first + npages) {
      first += npages;
      goff += (unsigned)len;
      ++s;
      fetch();
    }
    return s < nseq;
  }
};

}  // namespace glmkv
