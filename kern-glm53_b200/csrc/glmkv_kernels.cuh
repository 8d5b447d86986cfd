// The KV-cache path of GLM-5.3's prefill as sm_100a kernels. Every entry keeps the parameter list of
// the kern-glm53 glue kernel it replaces (source/glm_glue.cu), so a manifest binds it unchanged; the
// launch shapes (grid, block, dynamic shared memory) are this file's own and are listed with each
// entry. Included by exactly one translation unit per module (the shared library and the cubin).
#pragma once

#include "glmkv_device.cuh"

namespace glmkv {

__device__ unsigned int g_fault;  // FAULT_* bits, read and cleared by the host
constexpr uint64_t WAIT_LIMIT_NS = 1000000000ull;  // a bounded wait gives up after one second

// ================================================================================================ plan

constexpr int PLAN_THREADS = 256;
constexpr int PLAN_STAGED = 256;  // sequences whose cu / prefix a block keeps in shared memory

}  // namespace glmkv

// A row's sequence, position and indexer bounds (glm_glue.cu:105-125): s is the first sequence
// with s + 1 == nseq or cu[s + 1] > r, p = seq_lens[s] - (cu[s + 1] - r), ks the u32 sum of the
// lengths before s, ke = ks + p + 1, klen = p + 1, row_seq = s, zero = 0.
//   grid ceil(T / 256), block 256
extern "C" __global__ void __launch_bounds__(glmkv::PLAN_THREADS)
    glm_plan(const long long* __restrict__ cu, const int* __restrict__ seq_lens, int nseq, int* __restrict__ pos,
             unsigned* __restrict__ ks, unsigned* __restrict__ ke, int* __restrict__ klen, int* __restrict__ row_seq,
             int* __restrict__ zero, int T) {
  using namespace glmkv;
  __shared__ long long s_cu[PLAN_STAGED + 1];
  __shared__ unsigned s_off[PLAN_STAGED + 1];
  __shared__ int s_len[PLAN_STAGED];
  pdl_trigger();
  pdl_wait();
  const int staged = nseq < PLAN_STAGED ? (nseq > 0 ? nseq : 1) : PLAN_STAGED;
  for (int i = threadIdx.x; i < staged; i += blockDim.x) {
    s_cu[i + 1] = cu[i + 1];
    s_len[i] = seq_lens[i];
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // u32 prefix of the lengths, as the reference accumulates it
    unsigned o = 0;
    for (int i = 0; i < staged; ++i) {
      s_off[i] = o;
      o += (unsigned)s_len[i];
    }
    s_off[staged] = o;
  }
  __syncthreads();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= T) return;
  int s = 0;
  while (s + 1 < nseq && s + 1 < staged && s_cu[s + 1] <= r) ++s;
  unsigned goff = s_off[s];
  long long cnext = s_cu[s + 1];
  int len = s_len[s];
  if (s + 1 == staged && staged < nseq) {  // more sequences than staged: continue in global memory
    while (s + 1 < nseq && cu[s + 1] <= r) goff += (unsigned)seq_lens[s++];
    cnext = cu[s + 1];
    len = seq_lens[s];
  }
  const int p = len - (int)(cnext - r);
  pos[r] = p;
  ks[r] = goff;
  ke[r] = goff + (unsigned)p + 1u;
  klen[r] = p + 1;
  row_seq[r] = s;
  zero[r] = 0;
}

// ================================================================================================ prep

namespace glmkv {

constexpr int PREP_WARPS = 8;                            // a CTA: 8 warps, each its own rows
constexpr int PREP_THREADS = 32 * PREP_WARPS;
constexpr int PREP_BUFS = 2;                             // rows a warp holds in shared memory
constexpr int PREP_ROW = 2 * (QL + KVL + 2 * HALF + ID); // 5504 B: one [q_a | kv_a | k_pe | wk] row
constexpr int PREP_WGT = 4 * (QL + KVL + 2 * ID);        // f32 g_q | g_kv | ik_w | ik_b
constexpr int PREP_SMEM = PREP_WGT + PREP_WARPS * PREP_BUFS * PREP_ROW;

// Packed f32 pairs on Blackwell's f32x2 pipe: each half rounded exactly like the scalar operation.
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;"
      : "=l"(d)
      : "l"(*reinterpret_cast<const unsigned long long*>(&a)), "l"(*reinterpret_cast<const unsigned long long*>(&b)));
  return *reinterpret_cast<const float2*>(&d);
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(d)
      : "l"(*reinterpret_cast<const unsigned long long*>(&a)), "l"(*reinterpret_cast<const unsigned long long*>(&b)),
        "l"(*reinterpret_cast<const unsigned long long*>(&c)));
  return *reinterpret_cast<const float2*>(&d);
}
__device__ __forceinline__ float2 unpack2(uint32_t w) { return make_float2(bf_lo(w), bf_hi(w)); }
__device__ __forceinline__ uint32_t round2(float2 v) { return pack_bf16x2(v.x, v.y); }
// max(|a|, |b|) of two bf16 values in one word, as f32 (exact: bf16 compares exactly)
__device__ __forceinline__ float absmax_bf16x2(uint32_t w) {
  return fmaxf(fabsf(bf_lo(w)), fabsf(bf_hi(w)));
}
__device__ __forceinline__ uint32_t absmax2_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a & 0x7fff7fffu), "r"(b & 0x7fff7fffu));
  return d;
}

// max(|a|, |b|) per bf16 half, with the sign bit the xor of the operands' (callers mask it off).
__device__ __forceinline__ uint32_t absmax_xs(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// bf16x2 add and multiply, each half rounded once from the exact result (sm_90+).
__device__ __forceinline__ uint32_t add_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// Max over the warp of eight per-lane bf16x2 words (xorsign-abs max), scattered: lane l returns
// word (l >> 2) & 7.
__device__ __forceinline__ uint32_t max8w_scatter(const uint32_t (&v)[8], int l) {
  const bool b4 = l & 16, b3 = l & 8, b2 = l & 4;
  uint32_t a[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t send = b4 ? v[k] : v[k + 4], keep = b4 ? v[k + 4] : v[k];
    a[k] = absmax_xs(keep, __shfl_xor_sync(FULL, send, 16));
  }
  uint32_t b[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const uint32_t send = b3 ? a[k] : a[k + 2], keep = b3 ? a[k + 2] : a[k];
    b[k] = absmax_xs(keep, __shfl_xor_sync(FULL, send, 8));
  }
  const uint32_t send = b2 ? b[0] : b[1], keep = b2 ? b[1] : b[0];
  uint32_t c = absmax_xs(keep, __shfl_xor_sync(FULL, send, 4));
  c = absmax_xs(c, __shfl_xor_sync(FULL, c, 2));
  return absmax_xs(c, __shfl_xor_sync(FULL, c, 1));
}

// acc + w0^2 + w1^2 + w2^2 + w3^2 for the four bf16 values of v, in that order, each step one f32
// FMA of the bf16 operands (fma.rn.f32.bf16: the product is exact, so it rounds like fmaf on the
// widened values).
__device__ __forceinline__ float sq_acc4(uint2 v, float acc) {
  float d;
  asm("{\n\t.reg .b16 a, b, c, d;\n\t"
      "mov.b32 {a, b}, %1;\n\tmov.b32 {c, d}, %2;\n\t"
      "fma.rn.f32.bf16 %0, a, a, %3;\n\tfma.rn.f32.bf16 %0, b, b, %0;\n\t"
      "fma.rn.f32.bf16 %0, c, c, %0;\n\tfma.rn.f32.bf16 %0, d, d, %0;\n\t}"
      : "=f"(d)
      : "r"(v.x), "r"(v.y), "f"(acc));
  return d;
}

// The two bf16 values of w times s, as f32: one fma.rn.f32.bf16 each, whose addend -0 keeps the sign
// of a zero product, so each rounds like the f32 multiply of the widened value. s is the f32 bit
// pattern of a power of two (or 0 or inf) at least 2^-133: its low 16 bits are zero, so its high
// half is the same number as a bf16.
__device__ __forceinline__ float2 scale_bf16x2(uint32_t w, uint32_t s) {
  float2 d;
  asm("{\n\t.reg .b16 a, b, sl, sh;\n\t"
      "mov.b32 {a, b}, %2;\n\tmov.b32 {sl, sh}, %3;\n\t"
      "fma.rn.f32.bf16 %0, a, sh, 0f80000000;\n\tfma.rn.f32.bf16 %1, b, sh, 0f80000000;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "r"(w), "r"(s));
  return d;
}

// A row's operands: the warp's shared-memory copy, or global memory when the row is not 16-byte
// aligned for a bulk copy.
struct SmemRow {
  const u8* p;
  __device__ __forceinline__ uint2 v2(int off) const { return *reinterpret_cast<const uint2*>(p + off); }
  __device__ __forceinline__ uint32_t u32(int off) const { return *reinterpret_cast<const uint32_t*>(p + off); }
};
struct GlobalRow {
  const u8* p;
  __device__ __forceinline__ uint2 v2(int off) const { return ld_stream_v2(p + off); }
  __device__ __forceinline__ uint32_t u32(int off) const { return ld_stream_u32(p + off); }
};

// One row of the latent-cache append (glm_glue.cu:196-287), run by ONE warp. Lane l holds exactly
// the operands the reference's thread (w, l) holds for every warp w of its 256-thread block, so
// the RMS sums are built in the reference's order (block_sum8); everything else is per element or
// a max, which any order computes exactly. Weights come from shared memory as f32.
template <bool FP8, class Row>
__device__ __forceinline__ void prep_row(const Row& row, const float* __restrict__ wq, const float* __restrict__ wkv,
                                         const float* __restrict__ wik, const float* __restrict__ wib,
                                         const bf16* __restrict__ rope, int p, long long s, u8* __restrict__ kv,
                                         u8* __restrict__ idx, u8* __restrict__ qq, u8* __restrict__ qsf, int sf_rows,
                                         int r, int l, uint32_t* __restrict__ xw) {
  uint2 qw[16];  // q_a columns kb * 128 + 4l .. + 3
#pragma unroll
  for (int kb = 0; kb < 16; ++kb) qw[kb] = row.v2(2 * (kb * 128 + 4 * l));
  uint32_t kvw[8];  // kv_a columns 64w + 2l, + 1 (the reference's thread 32w + l)
#pragma unroll
  for (int w = 0; w < 8; ++w) kvw[w] = row.u32(2 * (QL + 64 * w + 2 * l));
  uint32_t csw = 0;  // rope[pos]: cs[2l], cs[2l + 1]
  if (s >= 0) csw = __ldg(reinterpret_cast<const unsigned*>(rope + (size_t)p * 2 * HALF) + l);

  // ---- RMS factors (glm_glue.cu:212-221): per-thread sequential partials, block_sum order. Virtual
  // warp h sums its blocks 2h and 2h + 1 in column order, one FMA of the bf16 operands a value.
  float part[8];
#pragma unroll
  for (int h = 0; h < 8; ++h) part[h] = sq_acc4(qw[2 * h + 1], sq_acc4(qw[2 * h], 0.f));
  const float rq = rsqrtf(block_sum8(part, l) / 2048.f + EPS);
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    const float2 a = make_float2(bf_lo(kvw[2 * h]), bf_lo(kvw[2 * h + 1]));
    const float2 b = make_float2(bf_hi(kvw[2 * h]), bf_hi(kvw[2 * h + 1]));
    const float2 t = fma2(a, a, mul2(b, b));  // both squares exact: round(a^2 + b^2)
    part[2 * h] = t.x, part[2 * h + 1] = t.y;
  }
  const float rk = rsqrtf(block_sum8(part, l) / 512.f + EPS);

  // ---- q_c = bf16((q_a * rq) * g_q), e4m3 per 128 columns with UE8M0 scales (glm_glue.cu:222-230)
  const float2 rq2 = make_float2(rq, rq);
  uint32_t yb[16][2];
#pragma unroll
  for (int kb = 0; kb < 16; ++kb) {
    const float4 g = *reinterpret_cast<const float4*>(wq + kb * 128 + 4 * l);
    yb[kb][0] = round2(mul2(mul2(unpack2(qw[kb].x), rq2), make_float2(g.x, g.y)));
    yb[kb][1] = round2(mul2(mul2(unpack2(qw[kb].y), rq2), make_float2(g.z, g.w)));
  }
  // |max| of this lane's values of blocks 2j (low half) and 2j + 1 (high half), then over the warp
  uint32_t m2[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t a = absmax_xs(yb[2 * j][0], yb[2 * j][1]), b = absmax_xs(yb[2 * j + 1][0], yb[2 * j + 1][1]);
    m2[j] = absmax_xs(__byte_perm(a, b, 0x5410), __byte_perm(a, b, 0x7632));
  }
  const uint32_t mw = max8w_scatter(m2, l);  // lane l: blocks 2 ((l >> 2) & 7) and 2 ((l >> 2) & 7) + 1
  const float bm = __uint_as_float(((l & 1) ? (mw & 0xffff0000u) : (mw << 16)) & 0x7fffffffu);
  unsigned e;
  const float inv = __frcp_rn(ue8m0_div(bm, 1e-10f, &e));  // lane l: block 2 ((l >> 2) & 7) + (l & 1)
  // Every block's inverse and UE8M0 byte reach the whole warp through its scratch words (one store and
  // four broadcast loads instead of 16 shuffles): word kb the inverse of block kb, byte 64 + kb its
  // scale byte, so that word 16 + q is DeepGEMM's packed word q (byte kb & 3 of word kb >> 2).
  __syncwarp();  // the previous row's reads of the scratch are done
  if ((l & 2) == 0) {
    const int blk = 2 * ((l >> 2) & 7) + (l & 1);
    xw[blk] = __float_as_uint(inv);
    reinterpret_cast<u8*>(xw + 16)[blk] = (u8)e;
  }
  __syncwarp();
  u8* qrow = qq + (size_t)r * QL;
#pragma unroll
  for (int k4 = 0; k4 < 16; k4 += 4) {
    const uint4 i4 = *reinterpret_cast<const uint4*>(xw + k4);
    const uint32_t ivs[4] = {i4.x, i4.y, i4.z, i4.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int kb = k4 + j;
      const float2 a = scale_bf16x2(yb[kb][0], ivs[j]), b = scale_bf16x2(yb[kb][1], ivs[j]);
      *reinterpret_cast<uint32_t*>(qrow + kb * 128 + 4 * l) = fp8x4(a.x, a.y, b.x, b.y);
    }
  }
  if (l < 4) *reinterpret_cast<unsigned*>(qsf + ((size_t)l * sf_rows + r) * 4) = xw[16 + l];

  if (s < 0) return;  // no cache slot: nothing more to write (glm_glue.cu:231-232)

  // ---- kv_norm = bf16((kv_a * rk) * g_kv) (glm_glue.cu:235), one bf16 pair a virtual thread
  const float2 rk2 = make_float2(rk, rk);
  uint32_t kn[8];
#pragma unroll
  for (int w = 0; w < 8; ++w)
    kn[w] = round2(mul2(mul2(unpack2(kvw[w]), rk2), *reinterpret_cast<const float2*>(wkv + 64 * w + 2 * l)));
  u8* dst = kv + s * (FP8 ? KV8 : KVB);
  if constexpr (FP8) {
    // tiles of 128 (two virtual warps), scale amax / 448, e4m3 satfinite (glm_glue.cu:238-247)
    // |max| per bf16 half of tile t (virtual warps 2t, 2t + 1); tiles 0 | 1 and 2 | 3 share a word,
    // which a reduce-scatter over the warp leaves in lanes < 16 and >= 16.
    const uint32_t t0 = absmax_xs(kn[0], kn[1]), t1 = absmax_xs(kn[2], kn[3]);
    const uint32_t t2 = absmax_xs(kn[4], kn[5]), t3 = absmax_xs(kn[6], kn[7]);
    const uint32_t p01 = absmax_xs(__byte_perm(t0, t1, 0x5410), __byte_perm(t0, t1, 0x7632));
    const uint32_t p23 = absmax_xs(__byte_perm(t2, t3, 0x5410), __byte_perm(t2, t3, 0x7632));
    const bool b4 = l & 16;
    uint32_t m = absmax_xs(b4 ? p23 : p01, __shfl_xor_sync(FULL, b4 ? p01 : p23, 16));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) m = absmax_xs(m, __shfl_xor_sync(FULL, m, o));
    // lane l: tile 2 (l >> 4) + (l & 1)
    const float tm = __uint_as_float(((l & 1) ? (m & 0xffff0000u) : (m << 16)) & 0x7fffffffu);
    const float sc = __fdiv_rn(tm, 448.f);
    const float tinv = sc > 0.f ? __frcp_rn(sc) : 0.f;
    // each tile's inverse and scale through the scratch as well: words 20 + t and 24 + t
    if ((l & 14) == 0) {
      const int t = 2 * (l >> 4) + (l & 1);
      xw[20 + t] = __float_as_uint(tinv);
      xw[24 + t] = __float_as_uint(sc);
    }
    __syncwarp();
    const uint4 t4 = *reinterpret_cast<const uint4*>(xw + 20);
    const float tiv[4] = {__uint_as_float(t4.x), __uint_as_float(t4.y), __uint_as_float(t4.z), __uint_as_float(t4.w)};
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const float iv = tiv[w >> 1];  // virtual warp w is in tile w / 2
      const float2 q = mul2(unpack2(kn[w]), make_float2(iv, iv));
      *reinterpret_cast<uint16_t*>(dst + 2 * (32 * w + l)) = fp8x2(q.x, q.y);
    }
    if (l < 4) reinterpret_cast<uint32_t*>(dst + KVL)[l] = xw[24 + l];
  } else {
#pragma unroll
    for (int w = 0; w < 8; ++w) *reinterpret_cast<uint32_t*>(dst + 4 * (32 * w + l)) = kn[w];
  }

  // ---- k_pe rope, interleaved pairs (glm_glue.cu:252-257). The bf16 x bf16 products are exact in
  // f32, so this equals round(x1 c - x2 sn) however the reference contracted it.
  const uint32_t pew = row.u32(2 * (QL + KVL + 2 * l));
  const uint32_t ca = __shfl_sync(FULL, csw, l >> 1), cb = __shfl_sync(FULL, csw, 16 + (l >> 1));
  {
    const float c = (l & 1) ? bf_hi(ca) : bf_lo(ca), sn = (l & 1) ? bf_hi(cb) : bf_lo(cb);
    const float x1 = bf_lo(pew), x2 = bf_hi(pew);
    *reinterpret_cast<uint32_t*>(dst + (FP8 ? KVL + 16 : 2 * KVL) + 4 * l) =
        pack_bf16x2(__fmaf_rn(x1, c, -__fmul_rn(x2, sn)), __fmaf_rn(x2, c, __fmul_rn(x1, sn)));
  }

  // ---- indexer key (glm_glue.cu:258-286): LayerNorm (eps 1e-6), rope on dims 0..63, UE8M0 e4m3
  if (idx == nullptr) return;
  const uint2 wkw = row.v2(2 * (QL + KVL + 2 * HALF + 4 * l));  // wk columns 4l .. + 3
  const float4 kw = *reinterpret_cast<const float4*>(wik + 4 * l);
  const float4 kbias = *reinterpret_cast<const float4*>(wib + 4 * l);
  const float k[4] = {bf_lo(wkw.x), bf_hi(wkw.x), bf_lo(wkw.y), bf_hi(wkw.y)};
  const float mean = warp_sum(((k[0] + k[1]) + k[2]) + k[3]) / 128.f;
  float d[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) d[j] = __fsub_rn(k[j], mean);
  // The f32 contractions of the reference's compiled code (found by running it on 2^20 rows against
  // every combination): d2 += d * d as one FMA a step; (d * rstd) * w + b with the last multiply
  // fused; the rope as fma(e, c, -(o * sn)) and fma(e, sn, o * c).
  float d2 = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) d2 = __fmaf_rn(d[j], d[j], d2);
  const float rstd = rsqrtf(warp_sum(d2) / 128.f + 1e-6f);
  float n[4] = {__fmaf_rn(__fmul_rn(d[0], rstd), kw.x, kbias.x), __fmaf_rn(__fmul_rn(d[1], rstd), kw.y, kbias.y),
                __fmaf_rn(__fmul_rn(d[2], rstd), kw.z, kbias.z), __fmaf_rn(__fmul_rn(d[3], rstd), kw.w, kbias.w)};
  const uint32_t csh = __shfl_sync(FULL, csw, (l + 16) & 31);  // cs[32 + 2l], cs[33 + 2l]
  if (l < 16) {
#pragma unroll
    for (int j = 0; j < 4; j += 2) {
      const float c = j ? bf_hi(csw) : bf_lo(csw), sn = j ? bf_hi(csh) : bf_lo(csh), ev = n[j], od = n[j + 1];
      n[j] = __fmaf_rn(ev, c, -__fmul_rn(od, sn));
      n[j + 1] = __fmaf_rn(ev, sn, __fmul_rn(od, c));
    }
  }
  const float amax = warp_max(fmaxf(fmaxf(fabsf(n[0]), fabsf(n[1])), fmaxf(fabsf(n[2]), fabsf(n[3]))));
  unsigned ex;
  const float sc = ue8m0(amax, 1e-4f, &ex), isc = ue8m0_inv(ex);  // n * (1 / sc) rounds as n / sc
  u8* page = idx + (size_t)(s / PAGE) * IDX_PAGE;
  const int i = (int)(s % PAGE);
  *reinterpret_cast<uint32_t*>(page + i * ID + 4 * l) =
      fp8x4(__fmul_rn(n[0], isc), __fmul_rn(n[1], isc), __fmul_rn(n[2], isc), __fmul_rn(n[3], isc));
  if (l == 0) reinterpret_cast<float*>(page + PAGE * ID)[i] = sc;
}

// The rows of a call, a warp at a time: warp g of the grid takes rows g, g + G, g + 2G, ... (G warps
// in the grid). While it works on one row, the next one is already on its way: a 1-D bulk copy
// (TMA) of the row's 5504 bytes (5248 on a shared layer, which has no wk) into the warp's other
// shared-memory buffer, completing on that buffer's mbarrier. Rows that are not 16-byte aligned
// (lda % 8 or x % 16) are read straight from global memory instead.
template <bool FP8>
__device__ __forceinline__ void prep_rows(const bf16* __restrict__ x, int lda, const bf16* __restrict__ g_q,
                                          const bf16* __restrict__ g_kv, const bf16* __restrict__ rope,
                                          const int* __restrict__ pos, const long long* __restrict__ slot,
                                          u8* __restrict__ kv, u8* __restrict__ idx, const bf16* __restrict__ ik_w,
                                          const bf16* __restrict__ ik_b, u8* __restrict__ qq, u8* __restrict__ qsf,
                                          int sf_rows, int T) {
  extern __shared__ __align__(128) u8 smem[];
  __shared__ __align__(8) unsigned long long bar[PREP_WARPS][PREP_BUFS];
  __shared__ __align__(16) uint32_t xws[PREP_WARPS][32];  // each warp's broadcast scratch (prep_row)
  float* wq = reinterpret_cast<float*>(smem);
  float* wkv = wq + QL;
  float* wik = wkv + KVL;
  float* wib = wik + ID;
  const int tid = threadIdx.x, warp = tid >> 5, l = tid & 31;
  if (l == 0) {
#pragma unroll
    for (int b = 0; b < PREP_BUFS; ++b) mbar_init(smem_u32(&bar[warp][b]), 1);
    mbar_init_fence();
  }
  pdl_trigger();  // a persistent grid: all of its CTAs are resident
  // The warp's first two rows into L2 before the wait: a prefetch is a hint that changes no value (L2 is
  // where the previous kernel's writes land), and it overlaps that kernel's drain (0.6% of the step).
  if (l == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (lda & 7) == 0) {
    const uint32_t nb = idx != nullptr ? PREP_ROW : 2 * (QL + MLA);
    const int r0 = blockIdx.x * PREP_WARPS + warp, st = gridDim.x * PREP_WARPS;
    if (r0 < T) prefetch_l2(x + (size_t)r0 * lda, nb);
    if (r0 + st < T) prefetch_l2(x + (size_t)(r0 + st) * lda, nb);
  }

  // The norm weights as f32, every load in flight at once (g_q and the indexer weights 8-byte aligned,
  // g_kv 4-byte aligned; the launcher checks). They are load-time weights that no kernel of the path
  // writes, so they are staged before the wait for the previous kernel on the stream: under
  // programmatic dependent launch this overlaps that kernel's tail.
  {
    const uint2 q0 = __ldg(reinterpret_cast<const uint2*>(g_q) + tid);
    const uint2 q1 = __ldg(reinterpret_cast<const uint2*>(g_q) + PREP_THREADS + tid);
    const uint32_t k0 = __ldg(reinterpret_cast<const unsigned*>(g_kv) + tid);
    const bool wi = idx != nullptr && tid < ID / 2;
    uint2 w = make_uint2(0u, 0u);
    if (wi) w = __ldg(reinterpret_cast<const uint2*>(tid < ID / 4 ? ik_w : ik_b) + (tid & (ID / 4 - 1)));
    static_assert(QL == 8 * PREP_THREADS && KVL == 2 * PREP_THREADS, "one pass of loads stages g_q and g_kv");
    *reinterpret_cast<float4*>(wq + 4 * tid) = make_float4(bf_lo(q0.x), bf_hi(q0.x), bf_lo(q0.y), bf_hi(q0.y));
    *reinterpret_cast<float4*>(wq + 4 * (PREP_THREADS + tid)) =
        make_float4(bf_lo(q1.x), bf_hi(q1.x), bf_lo(q1.y), bf_hi(q1.y));
    *reinterpret_cast<float2*>(wkv + 2 * tid) = make_float2(bf_lo(k0), bf_hi(k0));
    if (wi)
      *reinterpret_cast<float4*>((tid < ID / 4 ? wik : wib) + 4 * (tid & (ID / 4 - 1))) =
          make_float4(bf_lo(w.x), bf_hi(w.x), bf_lo(w.y), bf_hi(w.y));
  }
  pdl_wait();  // x, pos and slot come from the kernels before this one

  const int stride = gridDim.x * PREP_WARPS;
  int r = blockIdx.x * PREP_WARPS + warp;
  const bool bulk = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (lda & 7) == 0;
  const uint32_t bytes = idx != nullptr ? PREP_ROW : 2 * (QL + MLA);
  u8* buf = smem + PREP_WGT + (size_t)warp * PREP_BUFS * PREP_ROW;
  auto issue = [&](int b, int row) {
    const uint32_t mb = smem_u32(&bar[warp][b]);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_arrive_expect_tx(mb, bytes);
    tma_load_1d(smem_u32(buf + b * PREP_ROW), x + (size_t)row * lda, bytes, mb);
  };
  if (bulk && r < T && l == 0) issue(0, r);
  __syncthreads();

  if (r >= T) return;
  if (!bulk) {
    for (; r < T; r += stride)
      prep_row<FP8>(GlobalRow{reinterpret_cast<const u8*>(x + (size_t)r * lda)}, wq, wkv, wik, wib, rope, pos[r],
                    slot[r], kv, idx, qq, qsf, sf_rows, r, l, xws[warp]);
    return;
  }
  int p = pos[r];
  long long s = slot[r];
  for (int k = 0; r < T; ++k, r += stride) {
    const int b = k & 1, rn = r + stride;
    if (rn < T && l == 0) issue(b ^ 1, rn);  // that buffer's previous row is done (__syncwarp below)
    int pn = 0;  // the next row's position and slot, in flight while this row is worked on
    long long sn = -1;
    if (rn < T) pn = pos[rn], sn = slot[rn];
    const bool ok = mbar_wait_bounded(smem_u32(&bar[warp][b]), (uint32_t)((k >> 1) & 1), WAIT_LIMIT_NS);
    if (__any_sync(FULL, !ok)) {
      // A copy never completed: flag it, wait (bounded) for the warp's copies in flight, and return.
      if (l == 0) {
        atomicOr(&g_fault, FAULT_WAIT_TIMEOUT);
        if (rn < T)
          mbar_wait_bounded(smem_u32(&bar[warp][b ^ 1]), (uint32_t)(((k + 1) >> 1) & 1), WAIT_LIMIT_NS);
      }
      return;
    }
    prep_row<FP8>(SmemRow{buf + b * PREP_ROW}, wq, wkv, wik, wib, rope, p, s, kv, idx, qq, qsf, sf_rows, r, l,
                  xws[warp]);
    __syncwarp();
    p = pn, s = sn;
  }
}

}  // namespace glmkv

#define GLMKV_PREP_PARAMS                                                                                       \
  const glmkv::bf16 *__restrict__ x, int lda, const glmkv::bf16 *__restrict__ g_q,                            \
      const glmkv::bf16 *__restrict__ g_kv, const glmkv::bf16 *__restrict__ rope, const int *__restrict__ pos,  \
      const long long *__restrict__ slot, glmkv::u8 *__restrict__ kv, glmkv::u8 *__restrict__ idx,             \
      const glmkv::bf16 *__restrict__ ik_w, const glmkv::bf16 *__restrict__ ik_b, glmkv::u8 *__restrict__ qq, \
      glmkv::u8 *__restrict__ qsf, int sf_rows, int T
#define GLMKV_PREP_ARGS x, lda, g_q, g_kv, rope, pos, slot, kv, idx, ik_w, ik_b, qq, qsf, sf_rows, T

// `--kv bf16` append: row at kv + slot * 1152 (glm_glue.cu:294-296).
//   persistent: grid = SMs x resident CTAs, block 256, dynamic smem PREP_SMEM (99,328 B)
extern "C" __global__ void __launch_bounds__(glmkv::PREP_THREADS, 2) glm_mla_prep(GLMKV_PREP_PARAMS) {
  glmkv::prep_rows<false>(GLMKV_PREP_ARGS);
}
// fp8_ds_mla append: row at kv + slot * 656 (glm_glue.cu:297-299).
//   persistent: grid = SMs x resident CTAs, block 256, dynamic smem PREP_SMEM (99,328 B)
extern "C" __global__ void __launch_bounds__(glmkv::PREP_THREADS, 2) glm_mla_prep_fp8(GLMKV_PREP_PARAMS) {
  glmkv::prep_rows<true>(GLMKV_PREP_ARGS);
}

// ================================================================================================ page pipeline

namespace glmkv {

struct StageMeta {
  unsigned long long row;  // first stream row of the page
  unsigned long long sel;  // the page's rows to produce (bit i: row i)
  int n;                   // live rows in the page
  int first;               // the first row staged (the stage holds rows first .. of the page)
  int live;                // 0: past the last page, 1: loaded, 2: skipped (invalid page number), 3: no row wanted
};

// A persistent CTA walks the pages b, b + G, b + 2G, ... (G = gridDim.x) of the call's sequences.
// Thread 0 keeps NSTAGE pages in flight, each one bulk copy (TMA) of the page's bytes into its
// own shared-memory stage; all threads convert a stage once its mbarrier completes, then thread 0
// refills it with the CTA's next page. `Op` turns a staged page into its stream rows. An Op with
// SELECTIVE set names the rows of a page it wants (`select`): a page with none is neither read nor
// written, and only the span from its first to its last wanted row is copied.
template <int NT, int NSTAGE, class Op>
__device__ __forceinline__ void page_pipeline(const u8* __restrict__ state, const int* __restrict__ block_table,
                                              int max_pages, const int* __restrict__ seq_lens, int nseq, const Op& op) {
  extern __shared__ __align__(128) u8 smem[];
  __shared__ __align__(8) unsigned long long full[NSTAGE];
  __shared__ StageMeta meta[NSTAGE];
  const int tid = threadIdx.x;
  PageCursor cur;
  unsigned pending = 0, pend_parity = 0;  // thread 0: stages with a copy in flight, and its phase

  auto issue = [&](long long k) {
    const int st = (int)(k % NSTAGE);
    const uint32_t bar = smem_u32(&full[st]);
    const long long g = (long long)blockIdx.x + k * (long long)gridDim.x;
    if (!cur.seek(g)) {
      meta[st].live = 0;
      mbar_arrive(bar);
      return;
    }
    const int j = (int)(g - cur.first);
    const int n = min(PAGE, cur.len - j * PAGE);
    const unsigned long long row0 = (unsigned long long)cur.goff + (unsigned long long)j * PAGE;
    meta[st].row = row0;
    meta[st].n = n;
    int first = 0, count = n;
    if constexpr (Op::SELECTIVE) {
      const unsigned long long sel = op.select(row0, n);
      meta[st].sel = sel;
      if (sel == 0) {  // no row of this page is wanted: nothing to read or write
        meta[st].live = 3;
        mbar_arrive(bar);
        return;
      }
      first = __ffsll((long long)sel) - 1;
      count = 64 - __clzll((long long)sel) - first;
    }
    meta[st].first = first;
    const int phys = block_table[(size_t)cur.s * max_pages + j];
    if (phys < 0) {  // not a page of the state: skip it and flag the call
      meta[st].live = 2;
      atomicOr(&g_fault, FAULT_BAD_PAGE);
      mbar_arrive(bar);
      return;
    }
    meta[st].live = 1;
    const uint32_t bytes = Op::load_bytes(count);
    mbar_arrive_expect_tx(bar, bytes);
    tma_load_1d(smem_u32(smem + (size_t)st * Op::STAGE),
                state + (size_t)phys * Op::PAGE_BYTES + (size_t)first * Op::ROW_BYTES, bytes, bar);
    pending |= 1u << st;
    if ((k / NSTAGE) & 1) pend_parity |= 1u << st;
    else pend_parity &= ~(1u << st);
  };

  if (tid == 0) {
#pragma unroll
    for (int st = 0; st < NSTAGE; ++st) mbar_init(smem_u32(&full[st]), 1);
    mbar_init_fence();
  }
  pdl_trigger();  // a persistent grid: all of its CTAs are resident
  pdl_wait();
  if (tid == 0) cur.init(seq_lens, nseq);
  __syncthreads();
  if (tid == 0)
    for (int k = 0; k < NSTAGE; ++k) issue(k);

  for (long long k = 0;; ++k) {
    const int st = (int)(k % NSTAGE);
    const bool ok = mbar_wait_bounded(smem_u32(&full[st]), (uint32_t)((k / NSTAGE) & 1), WAIT_LIMIT_NS);
    if (__syncthreads_or(!ok)) {
      // A copy never completed: flag it, wait (bounded) for copies still in flight, and return.
      if (tid == 0) {
        atomicOr(&g_fault, FAULT_WAIT_TIMEOUT);
        for (int q = 0; q < NSTAGE; ++q)
          if (pending & (1u << q)) mbar_wait_bounded(smem_u32(&full[q]), (pend_parity >> q) & 1u, WAIT_LIMIT_NS);
      }
      return;
    }
    const StageMeta m = meta[st];
    if (m.live == 0) break;
    if (tid == 0) pending &= ~(1u << st);
    if (m.live == 1) {
      if constexpr (Op::SELECTIVE)
        op.template consume_sel<NT>(smem + (size_t)st * Op::STAGE, m.row, m.first, m.sel, tid);
      else
        op.template consume<NT>(smem + (size_t)st * Op::STAGE, m.row, m.n, tid);
    }
    __syncthreads();
    if (tid == 0) issue(k + NSTAGE);
  }
}

// ------------------------------------------------------------------------------------------------ dequant

constexpr int DQ_THREADS = 512;
constexpr int DQ_STAGES = 4;

struct DequantOp {
  static constexpr int STAGE = KV8_PAGE;
  static constexpr int PAGE_BYTES = KV8_PAGE;
  static constexpr int ROW_BYTES = KV8;
  static constexpr bool SELECTIVE = false;
  bf16* kvd;
  __device__ static uint32_t load_bytes(int n) { return (uint32_t)n * KV8; }

  // Rows [0, n) of a staged page -> stream rows row0 .. row0 + n of kvd [., 576]: every e4m3 byte
  // times its tile's f32 scale, rounded to bf16; k_pe's 128 bytes as they are (glm_glue.cu:396-413).
  template <int NT>
  __device__ __forceinline__ void consume(const u8* __restrict__ stg, unsigned long long row0, int n, int tid) const {
    u8* out = reinterpret_cast<u8*>(kvd) + row0 * KVB;
    const int nkv = n << 6;  // 16-byte output chunks of kv_norm: 64 a row
#pragma unroll 4
    for (int i = tid; i < nkv; i += NT) {
      const int r = i >> 6, c = i & 63;
      const u8* src = stg + r * KV8;
      const uint2 q = *reinterpret_cast<const uint2*>(src + 8 * c);
      const float sc = reinterpret_cast<const float*>(src + KVL)[c >> 4];
      uint4 o;
      o.x = dequant2((uint16_t)(q.x & 0xffffu), sc);
      o.y = dequant2((uint16_t)(q.x >> 16), sc);
      o.z = dequant2((uint16_t)(q.y & 0xffffu), sc);
      o.w = dequant2((uint16_t)(q.y >> 16), sc);
      *reinterpret_cast<uint4*>(out + (size_t)r * KVB + 16 * c) = o;
    }
    const int npe = n << 3;  // k_pe: 8 chunks a row
    for (int i = tid; i < npe; i += NT) {
      const int r = i >> 3, c = i & 7;
      *reinterpret_cast<uint4*>(out + (size_t)r * KVB + 2 * KVL + 16 * c) =
          *reinterpret_cast<const uint4*>(stg + r * KV8 + KVL + 16 + 16 * c);
    }
  }
};

// ------------------------------------------------------------------------------------------------ gather

// 6 stages a CTA, so that 4 CTAs fit an SM (24 pages in flight): measured against 3 CTAs of 8 and
// 5, 6 or 8 CTAs of fewer stages, the one shape faster at both 16,384 rows over 549K tokens and 1M
constexpr int GA_THREADS = 256;
constexpr int GA_STAGES = 6;

struct GatherOp {
  static constexpr int STAGE = IDX_PAGE;
  static constexpr int PAGE_BYTES = IDX_PAGE;
  static constexpr int ROW_BYTES = 0;  // the whole page is one copy: keys and scales
  static constexpr bool SELECTIVE = false;
  u8* kg;
  float* ksf;
  __device__ static uint32_t load_bytes(int) { return IDX_PAGE; }  // keys and scales in one copy

  // Rows [0, n) of a staged index page -> kg rows row0 .. (128 bytes each) and ksf (glm_glue.cu:369-375).
  template <int NT>
  __device__ __forceinline__ void consume(const u8* __restrict__ stg, unsigned long long row0, int n, int tid) const {
    uint4* dst = reinterpret_cast<uint4*>(kg + row0 * ID);
    const uint4* src = reinterpret_cast<const uint4*>(stg);
    const int nk = n << 3;
#pragma unroll 2
    for (int i = tid; i < nk; i += NT) dst[i] = src[i];
    if (tid < n) ksf[row0 + tid] = reinterpret_cast<const float*>(stg + PAGE * ID)[tid];
  }
};

// ------------------------------------------------------------------------------------------------ marked dequant

// The dequant of only the stream rows a call's picks name. `mask` has a bit for every stream row
// (word w: rows 64 w .. 64 w + 63, bit i row 64 w + i), set by glm_mark_rows. Rows produce exactly
// the bytes of DequantOp; rows not marked are not written.
struct MarkedDequantOp : DequantOp {
  static constexpr bool SELECTIVE = true;
  const unsigned long long* mask;

  // the marked rows of the page whose n rows start at stream row row0 (bit i: row i of the page)
  __device__ __forceinline__ unsigned long long select(unsigned long long row0, int n) const {
    const unsigned long long w = row0 >> 6;
    const int b = (int)(row0 & 63);
    unsigned long long m = __ldg(mask + w) >> b;
    if (b != 0 && row0 + (unsigned long long)n > (w + 1) * 64) m |= __ldg(mask + w + 1) << (64 - b);
    return n == 64 ? m : m & ((1ull << n) - 1);
  }

  // the staged rows first .. 63 - clz(sel) of the page -> their stream rows, marked rows only
  template <int NT>
  __device__ __forceinline__ void consume_sel(const u8* __restrict__ stg, unsigned long long row0, int first,
                                              unsigned long long sel, int tid) const {
    u8* out = reinterpret_cast<u8*>(kvd) + row0 * KVB;
    const int count = 64 - __clzll((long long)sel) - first;
    const int nkv = count << 6;
#pragma unroll 4
    for (int i = tid; i < nkv; i += NT) {
      const int rr = i >> 6, c = i & 63, r = first + rr;
      if (!((sel >> r) & 1ull)) continue;
      const u8* src = stg + rr * KV8;
      const uint2 q = *reinterpret_cast<const uint2*>(src + 8 * c);
      const float sc = reinterpret_cast<const float*>(src + KVL)[c >> 4];
      uint4 o;
      o.x = dequant2((uint16_t)(q.x & 0xffffu), sc);
      o.y = dequant2((uint16_t)(q.x >> 16), sc);
      o.z = dequant2((uint16_t)(q.y & 0xffffu), sc);
      o.w = dequant2((uint16_t)(q.y >> 16), sc);
      *reinterpret_cast<uint4*>(out + (size_t)r * KVB + 16 * c) = o;
    }
    const int npe = count << 3;
    for (int i = tid; i < npe; i += NT) {
      const int rr = i >> 3, c = i & 7, r = first + rr;
      if (!((sel >> r) & 1ull)) continue;
      *reinterpret_cast<uint4*>(out + (size_t)r * KVB + 2 * KVL + 16 * c) =
          *reinterpret_cast<const uint4*>(stg + rr * KV8 + KVL + 16 + 16 * c);
    }
  }
};

// ------------------------------------------------------------------------------------------------ mark

// 1024 threads: the shared-memory atomics are latency-bound, so the CTA (one an SM: the window takes
// 128 KB) brings as many warps as it can; 256 threads took twice as long
constexpr int MK_THREADS = 1024;
constexpr int MK_RB = 8;                                  // rows of picks a loop iteration
constexpr int MK_LD = MK_RB * (TOPK / 4) / MK_THREADS;    // 16-byte loads a thread an iteration, all in flight
static_assert(MK_LD * MK_THREADS == MK_RB * (TOPK / 4), "an iteration's rows split evenly over the threads");
constexpr int MK_WORDS = (1 << 20) / 32 + 2;       // shared-memory window: a 2^20-row stream, unaligned
constexpr int MK_SMEM = MK_WORDS * 4;              // 131,080 B

// a sequence-relative pick as a row of the dequantized stream (glm_glue.cu:421-425): -1 stays -1
__device__ __forceinline__ int stream_row(int k, unsigned base) { return k < 0 ? -1 : (int)(base + (unsigned)k); }

// The body of glm_mark_rows and glm_topk_stream_mark: a CTA takes an equal run of rows [r0, r1), whose
// picks lie inside the stream rows [min ks, max ke) (glm_plan). It marks them in a window of shared
// memory (2^20 rows at most) with 32-bit atomics (a 64-bit shared-memory OR measured 8x slower), then
// ORs the window into mask word by word: one global atomic a word a CTA rather than one a pick. The
// mask is addressed as 32-bit words, which on this little-endian device is the same bitmap. A pick
// outside the window (malformed picks) is ORed straight into mask, and one past mask_words * 64 is
// skipped and flagged (fault bit 4). With REMAP the picks arrive sequence-relative (-1 past a short
// row's keys) and are first rewritten in place as the stream rows glm_topk_stream writes, with tlen
// as it writes it (glm_glue.cu:416-428), so that the row plan and the mark read the picks once.
template <bool REMAP>
__device__ __forceinline__ void mark_rows(int* __restrict__ ind, const unsigned* __restrict__ ks,
                                          const int* __restrict__ klen, int* __restrict__ tlen,
                                          const unsigned* __restrict__ ke, int T, unsigned long long* __restrict__ mask,
                                          int mask_words) {
  extern __shared__ __align__(16) unsigned win[];
  __shared__ unsigned s_lo[MK_THREADS / 32], s_hi[MK_THREADS / 32];
  pdl_trigger();
  pdl_wait();
  const int tid = threadIdx.x, l = tid & 31, w = tid >> 5;
  const int per = (T + (int)gridDim.x - 1) / (int)gridDim.x;
  const int r0 = min(T, (int)blockIdx.x * per), r1 = min(T, r0 + per);
  unsigned* const mask32 = reinterpret_cast<unsigned*>(mask);
  const long long words32 = 2ll * mask_words;
  // the window: the stream rows these rows' picks can name
  unsigned lo = 0xffffffffu, hi = 0u;
  for (int r = r0 + tid; r < r1; r += MK_THREADS) lo = min(lo, ks[r]), hi = max(hi, ke[r]);
  lo = __reduce_min_sync(FULL, lo);
  hi = __reduce_max_sync(FULL, hi);
  if (l == 0) s_lo[w] = lo, s_hi[w] = hi;
  __syncthreads();
  lo = 0xffffffffu, hi = 0u;
#pragma unroll
  for (int i = 0; i < MK_THREADS / 32; ++i) lo = min(lo, s_lo[i]), hi = max(hi, s_hi[i]);
  const long long wlo = lo >> 5;
  const long long whi = min(((long long)hi + 31) >> 5, words32);
  const int nw = whi > wlo ? (int)(whi - wlo) : 0;
  const bool windowed = nw <= MK_WORDS;
  if (windowed)
    for (int i = tid; i < nw; i += MK_THREADS) win[i] = 0u;
  __syncthreads();
  auto put = [&](int p) {
    if (p < 0) return;
    const long long wd = p >> 5;
    const unsigned bit = 1u << (p & 31);
    if (windowed && wd >= wlo && wd < whi) {
      atomicOr(&win[wd - wlo], bit);
    } else if (wd < words32) {
      atomicOr(mask32 + wd, bit);
    } else {
      atomicOr(&g_fault, FAULT_BAD_PICK);
    }
  };
  for (int r = r0; r < r1; r += MK_RB) {
    int4 v[MK_LD];
#pragma unroll
    for (int k = 0; k < MK_LD; ++k) {
      const int f = k * MK_THREADS + tid;  // 16-byte piece f of the MK_RB rows, row-major
      const int rr = r + f / (TOPK / 4);
      const int4* src = reinterpret_cast<const int4*>(ind + (size_t)rr * TOPK) + f % (TOPK / 4);
      if constexpr (REMAP)  // read, then rewritten below: a plain load, not the read-only path
        v[k] = rr < r1 ? *src : make_int4(-1, -1, -1, -1);
      else
        v[k] = rr < r1 ? ld_stream_v4(src) : make_int4(-1, -1, -1, -1);
    }
    if constexpr (REMAP) {
#pragma unroll
      for (int k = 0; k < MK_LD; ++k) {
        const int f = k * MK_THREADS + tid;
        const int rr = r + f / (TOPK / 4);
        if (rr < r1) {
          const unsigned base = ks[rr];
          v[k] = make_int4(stream_row(v[k].x, base), stream_row(v[k].y, base), stream_row(v[k].z, base),
                           stream_row(v[k].w, base));
          reinterpret_cast<int4*>(ind + (size_t)rr * TOPK)[f % (TOPK / 4)] = v[k];
        }
      }
    }
#pragma unroll
    for (int k = 0; k < MK_LD; ++k) put(v[k].x), put(v[k].y), put(v[k].z), put(v[k].w);
  }
  if constexpr (REMAP)
    for (int r = r0 + tid; r < r1; r += MK_THREADS) tlen[r] = min(klen[r], TOPK);
  __syncthreads();
  if (windowed)
    for (int i = tid; i < nw; i += MK_THREADS) {
      const unsigned m = win[i];
      if (m) atomicOr(mask32 + wlo + i, m);
    }
}

}  // namespace glmkv

// The stream rows a call's picks name, as a bitmap: bit p % 64 of word p / 64 for every pick p >= 0 of
// ind [T, 2048] (stream rows, after glm_topk_stream). The launcher clears mask first and sizes the
// grid so that every SM takes an equal run of rows (mark_rows above). No counterpart in the
// reference: it feeds glm_kv_dequant_marked.
//   grid min(SMs, ceil(T / 8)), block 1024, dynamic smem MK_SMEM (131,080 B)
extern "C" __global__ void __launch_bounds__(glmkv::MK_THREADS)
    glm_mark_rows(const int* __restrict__ ind, const unsigned* __restrict__ ks, const unsigned* __restrict__ ke,
                  int T, unsigned long long* __restrict__ mask, int mask_words) {
  glmkv::mark_rows<false>(const_cast<int*>(ind), ks, nullptr, nullptr, ke, T, mask, mask_words);
}

// glm_topk_stream and glm_mark_rows in one pass over the picks: ind [T, 2048] sequence-relative in,
// stream rows out (in place), tlen = min(klen, 2048), and the bitmap of the stream rows named. Its
// first five parameters are glm_topk_stream's; ke, mask and mask_words are glm_mark_rows'. No
// counterpart in the reference.
//   grid min(SMs, ceil(T / 8)), block 1024, dynamic smem MK_SMEM (131,080 B)
extern "C" __global__ void __launch_bounds__(glmkv::MK_THREADS)
    glm_topk_stream_mark(int* __restrict__ ind, const unsigned* __restrict__ ks, const int* __restrict__ klen,
                         int* __restrict__ tlen, int T, const unsigned* __restrict__ ke,
                         unsigned long long* __restrict__ mask, int mask_words) {
  glmkv::mark_rows<true>(ind, ks, klen, tlen, ke, T, mask, mask_words);
}

namespace glmkv {

constexpr int ML_SEQ = 1024;  // sequences a planned marked lift holds in shared memory (more: cursor walk)
constexpr int ML_CAP = 1024;  // pages a CTA plans at a time
constexpr int ML_DENSE = 48;  // a page with this many marked rows is lifted whole

struct MlEntry {
  unsigned long long row;  // first stream row of the page
  unsigned long long sel;  // its rows to produce (all of them for an Op that is not SELECTIVE)
  int phys;                // its page in the state
  int n;                   // its live rows
};

// A page pipeline with the CTA's pages planned up front, for the marked lift: all threads find, for a
// batch of the CTA's pages b, b + G, ... at once, each page's sequence (a binary search over the pages
// of the sequences before it), its marked rows and, when it has any, its page number; the pages with
// marked rows are compacted, in order, into a list. Thread 0 then streams the listed pages as
// page_pipeline does, so a page with no marked row costs a mask read and nothing else. A page with
// ML_DENSE or more marked rows is lifted whole (its other rows get the bytes the full lift writes
// there): skipping a few rows of a page saves little and costs the page's even run of stores. Needs
// nseq <= ML_SEQ. (On the full lift, where no page is skipped, page_pipeline's cursor streams 15%
// faster: measured, not explained by its counters. So only the marked lift plans.)
template <int NT, int NSTAGE, class Op, int CAP = ML_CAP, int SEQ = ML_SEQ>
__device__ __forceinline__ void planned_pipeline(const u8* __restrict__ state, const int* __restrict__ block_table,
                                                 int max_pages, const int* __restrict__ seq_lens, int nseq,
                                                 const Op& op) {
  extern __shared__ __align__(128) u8 smem[];
  __shared__ __align__(8) unsigned long long full[NSTAGE];
  __shared__ MlEntry list[CAP];
  __shared__ int s_len[SEQ], s_pages[SEQ + 1];
  __shared__ unsigned s_goff[SEQ + 1];
  __shared__ int s_wsum[NT / 32], s_count;
  const int tid = threadIdx.x, l = tid & 31, w = tid >> 5;
  if (tid == 0) {
#pragma unroll
    for (int st = 0; st < NSTAGE; ++st) mbar_init(smem_u32(&full[st]), 1);
    mbar_init_fence();
  }
  pdl_trigger();  // a persistent grid: all of its CTAs are resident
  pdl_wait();
  // pages and rows of the sequences before each one: a block scan, NT sequences at a time
  int carry_pages = 0;
  unsigned carry_rows = 0;
  for (int base = 0; base < nseq; base += NT) {
    const int s = base + tid;
    const int len = s < nseq ? seq_lens[s] : 0;
    const int pg = (len + PAGE - 1) / PAGE;
    int ip = pg;
    unsigned ir = (unsigned)len;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int a = __shfl_up_sync(FULL, ip, o);
      const unsigned b = __shfl_up_sync(FULL, ir, o);
      if (l >= o) ip += a, ir += b;
    }
    __shared__ unsigned s_wrows[NT / 32];
    if (l == 31) s_wsum[w] = ip, s_wrows[w] = ir;
    __syncthreads();
    int wp = 0;
    unsigned wr = 0;
    for (int i = 0; i < w; ++i) wp += s_wsum[i], wr += s_wrows[i];
    if (s < nseq) {
      s_len[s] = len;
      s_pages[s] = carry_pages + wp + ip - pg;  // exclusive prefix
      s_goff[s] = carry_rows + wr + ir - (unsigned)len;
    }
    int tp = 0;
    unsigned tr = 0;
    for (int i = 0; i < NT / 32; ++i) tp += s_wsum[i], tr += s_wrows[i];
    carry_pages += tp, carry_rows += tr;
    __syncthreads();
  }
  if (tid == 0) s_pages[nseq] = carry_pages;
  __syncthreads();
  const long long total = carry_pages, G = gridDim.x;
  const long long mine = total > (long long)blockIdx.x ? (total - 1 - blockIdx.x) / G + 1 : 0;  // this CTA's pages

  long long k = 0;  // stage uses so far (their mbarrier phases)
  for (long long done = 0; done < mine; done += CAP) {
    // ---- plan: the next CAP of this CTA's pages, those with marked rows listed in order
    if (tid == 0) s_count = 0;
    __syncthreads();
    for (int b = 0; b < CAP && done + b < mine; b += NT) {
      const long long kk = done + b + tid;
      bool want = false;
      MlEntry e;
      if (b + tid < CAP && kk < mine) {
        const int g = (int)(blockIdx.x + kk * G);
        int lo = 0, hi = nseq - 1;  // the last sequence whose first page is <= g
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (s_pages[mid] <= g) lo = mid;
          else hi = mid - 1;
        }
        const int j = g - s_pages[lo];
        e.n = min(PAGE, s_len[lo] - j * PAGE);
        e.row = (unsigned long long)s_goff[lo] + (unsigned long long)j * PAGE;
        const unsigned long long all = e.n == 64 ? ~0ull : (1ull << e.n) - 1;
        if constexpr (Op::SELECTIVE) {
          e.sel = op.select(e.row, e.n);
          if (__popcll(e.sel) >= ML_DENSE) e.sel = all;  // lift it whole
        } else {
          e.sel = all;
        }
        want = e.sel != 0;
        if (want) e.phys = block_table[(size_t)lo * max_pages + j];
      }
      const unsigned bal = __ballot_sync(FULL, want);
      if (l == 0) s_wsum[w] = __popc(bal);
      __syncthreads();
      int off = 0;
      for (int i = 0; i < w; ++i) off += s_wsum[i];
      if (want) list[s_count + off + __popc(bal & ((1u << l) - 1))] = e;
      __syncthreads();
      if (tid == 0)
        for (int i = 0; i < NT / 32; ++i) s_count += s_wsum[i];
      __syncthreads();
    }
    const int count = s_count;
    // ---- stream the listed pages, NSTAGE in flight
    unsigned pending = 0, pend_parity = 0;
    auto issue = [&](int i) {  // list entry i into stage (k + i) % NSTAGE
      const long long u = k + i;
      const int st = (int)(u % NSTAGE);
      const uint32_t bar = smem_u32(&full[st]);
      if (i >= count) {
        mbar_arrive(bar);
        return;
      }
      const MlEntry& e = list[i];
      if (e.phys < 0) {  // not a page of the state: skip it and flag the call
        atomicOr(&g_fault, FAULT_BAD_PAGE);
        mbar_arrive(bar);
        return;
      }
      int first = 0, cnt = e.n;
      if constexpr (Op::SELECTIVE) first = __ffsll((long long)e.sel) - 1, cnt = 64 - __clzll((long long)e.sel) - first;
      const uint32_t bytes = Op::load_bytes(cnt);
      mbar_arrive_expect_tx(bar, bytes);
      tma_load_1d(smem_u32(smem + (size_t)st * Op::STAGE),
                  state + (size_t)e.phys * Op::PAGE_BYTES + (size_t)first * Op::ROW_BYTES, bytes, bar);
      pending |= 1u << st;
      if ((u / NSTAGE) & 1) pend_parity |= 1u << st;
      else pend_parity &= ~(1u << st);
    };
    if (tid == 0)
      for (int i = 0; i < NSTAGE; ++i) issue(i);
    for (int i = 0; i < count; ++i) {
      const long long u = k + i;
      const int st = (int)(u % NSTAGE);
      const bool ok = mbar_wait_bounded(smem_u32(&full[st]), (uint32_t)((u / NSTAGE) & 1), WAIT_LIMIT_NS);
      if (__syncthreads_or(!ok)) {
        if (tid == 0) {
          atomicOr(&g_fault, FAULT_WAIT_TIMEOUT);
          for (int q = 0; q < NSTAGE; ++q)
            if (pending & (1u << q)) mbar_wait_bounded(smem_u32(&full[q]), (pend_parity >> q) & 1u, WAIT_LIMIT_NS);
        }
        return;
      }
      if (tid == 0) pending &= ~(1u << st);
      const MlEntry e = list[i];
      if (e.phys >= 0) {
        if constexpr (Op::SELECTIVE)
          op.template consume_sel<NT>(smem + (size_t)st * Op::STAGE, e.row, __ffsll((long long)e.sel) - 1, e.sel,
                                      tid);
        else
          op.template consume<NT>(smem + (size_t)st * Op::STAGE, e.row, e.n, tid);
      }
      __syncthreads();
      if (tid == 0) issue(i + NSTAGE);
    }
    // the NSTAGE stages issued past the list's end completed on plain arrives: consume their phases
    for (int i = count; i < count + NSTAGE; ++i) {
      const long long u = k + i;
      mbar_wait_bounded(smem_u32(&full[(int)(u % NSTAGE)]), (uint32_t)((u / NSTAGE) & 1), WAIT_LIMIT_NS);
    }
    k += count + NSTAGE;
    __syncthreads();
  }
}

}  // namespace glmkv

// The stream of glm_kv_dequant restricted to the rows mask marks (glm_mark_rows): a marked row gets
// exactly the bytes glm_kv_dequant writes there; a page with no marked row is neither read nor
// written; a page with at least ML_DENSE (48) marked rows is lifted whole, as glm_kv_dequant lifts it;
// of the other pages only the span from the first to the last marked row is read and only the marked
// rows are written. (With more than ML_SEQ sequences the lift walks the pages with the cursor and
// writes marked rows only.) mask must hold ceil(stream / 64) words. No counterpart in the reference,
// whose lift converts every row (glm_glue.cu:378-414).
//   persistent: grid = SMs x resident CTAs, block 512, dynamic smem DQ_STAGES * 41984 B
extern "C" __global__ void __launch_bounds__(glmkv::DQ_THREADS, 1)
    glm_kv_dequant_marked(const glmkv::u8* __restrict__ kv, const int* __restrict__ block_table, int max_pages,
                          const int* __restrict__ seq_lens, int nseq, const unsigned long long* __restrict__ mask,
                          glmkv::bf16* __restrict__ kvd) {
  glmkv::MarkedDequantOp op;
  op.kvd = kvd;
  op.mask = mask;
  if (nseq <= glmkv::ML_SEQ)
    glmkv::planned_pipeline<glmkv::DQ_THREADS, glmkv::DQ_STAGES>(kv, block_table, max_pages, seq_lens, nseq, op);
  else
    glmkv::page_pipeline<glmkv::DQ_THREADS, glmkv::DQ_STAGES>(kv, block_table, max_pages, seq_lens, nseq, op);
}

// The indexer keys of every sequence back to back (glm_glue.cu:353-376): page j of sequence s lands
// at stream rows goff(s) + 64 j, keys in kg [., 128], scales in ksf.
//   persistent: grid = SMs x resident CTAs, block 256, dynamic smem GA_STAGES * 8448 B
extern "C" __global__ void __launch_bounds__(glmkv::GA_THREADS)
    glm_idx_gather(const glmkv::u8* __restrict__ idx, const int* __restrict__ block_table, int max_pages,
                   const int* __restrict__ seq_lens, int nseq, glmkv::u8* __restrict__ kg, float* __restrict__ ksf) {
  glmkv::page_pipeline<glmkv::GA_THREADS, glmkv::GA_STAGES>(idx, block_table, max_pages, seq_lens, nseq,
                                                            glmkv::GatherOp{kg, ksf});
}

// The fp8 latent rows of every sequence lifted to bf16 back to back, the stream of glm_idx_gather
// (glm_glue.cu:378-414).
//   persistent: grid = SMs x resident CTAs, block 512, dynamic smem DQ_STAGES * 41984 B
extern "C" __global__ void __launch_bounds__(glmkv::DQ_THREADS, 1)
    glm_kv_dequant(const glmkv::u8* __restrict__ kv, const int* __restrict__ block_table, int max_pages,
                   const int* __restrict__ seq_lens, int nseq, glmkv::bf16* __restrict__ kvd) {
  glmkv::page_pipeline<glmkv::DQ_THREADS, glmkv::DQ_STAGES>(kv, block_table, max_pages, seq_lens, nseq,
                                                            glmkv::DequantOp{kvd});
}

// ================================================================================================ row plans

namespace glmkv {
constexpr int TK_THREADS = 256;  // a row of 2048 indices: two int4 a thread

__device__ __forceinline__ int slot_of(int k, const int* __restrict__ bt) {
  return k < 0 ? -1 : bt[k >> 6] * PAGE + (k & (PAGE - 1));
}
}  // namespace glmkv

// Sequence-relative top-k picks (-1 past a short row's keys) -> rows of the dequantized stream, in
// place; tlen = min(klen, 2048) (glm_glue.cu:416-428).
//   grid T, block 256
extern "C" __global__ void __launch_bounds__(glmkv::TK_THREADS)
    glm_topk_stream(int* __restrict__ ind, const unsigned* __restrict__ ks, const int* __restrict__ klen,
                    int* __restrict__ tlen, int T) {
  using namespace glmkv;
  pdl_trigger();  // the next kernel may start once every CTA of this grid has started
  pdl_wait();
  const int r = blockIdx.x;
  int4* row = reinterpret_cast<int4*>(ind + (size_t)r * TOPK);
  const unsigned base = ks[r];
  for (int i = threadIdx.x; i < TOPK / 8; i += blockDim.x) {
    int4 a = row[i], b = row[i + TOPK / 8];
    a = make_int4(stream_row(a.x, base), stream_row(a.y, base), stream_row(a.z, base), stream_row(a.w, base));
    b = make_int4(stream_row(b.x, base), stream_row(b.y, base), stream_row(b.z, base), stream_row(b.w, base));
    row[i] = a;
    row[i + TOPK / 8] = b;
  }
  if (threadIdx.x == 0) tlen[r] = min(klen[r], TOPK);
}

// Sequence-relative top-k picks -> cache slots through the row's page table, in place; tlen as
// above (glm_glue.cu:430-444).
//   grid T, block 256
extern "C" __global__ void __launch_bounds__(glmkv::TK_THREADS)
    glm_topk_slots(int* __restrict__ ind, const int* __restrict__ block_table, int max_pages,
                   const int* __restrict__ row_seq, const int* __restrict__ klen, int* __restrict__ tlen, int T) {
  using namespace glmkv;
  pdl_trigger();  // the next kernel may start once every CTA of this grid has started
  pdl_wait();
  const int r = blockIdx.x;
  const int* bt = block_table + (size_t)row_seq[r] * max_pages;
  int4* row = reinterpret_cast<int4*>(ind + (size_t)r * TOPK);
  for (int i = threadIdx.x; i < TOPK / 8; i += blockDim.x) {
    int4 a = row[i], b = row[i + TOPK / 8];
    a = make_int4(slot_of(a.x, bt), slot_of(a.y, bt), slot_of(a.z, bt), slot_of(a.w, bt));
    b = make_int4(slot_of(b.x, bt), slot_of(b.y, bt), slot_of(b.z, bt), slot_of(b.w, bt));
    row[i] = a;
    row[i + TOPK / 8] = b;
  }
  if (threadIdx.x == 0) tlen[r] = min(klen[r], TOPK);
}

// ================================================================================================ q post

namespace glmkv {

constexpr int HEADS = 64, QHD = 256, NOPE = 192, IH = 32;
constexpr int QP_WARPS = 8;  // a CTA: 8 warps, one row each
constexpr int QP_THREADS = 32 * QP_WARPS;

// (x1 c - x2 s, x2 c + x1 s) of the bf16 pair w = (x1, x2), as bf16 RN, with c, s and -s the bf16
// in half H of cw, sw and nsw. Both products of each output are bf16 x bf16, exact in f32, so the
// mixed-precision FMAs round exactly as the reference's fmaf(x1, c, -(x2 * s)) and
// fmaf(x2, c, x1 * s) on widened values; the addend -0 keeps the sign of a zero product.
template <int H>
__device__ __forceinline__ uint32_t rope_bf16(uint32_t w, uint32_t cw, uint32_t sw, uint32_t nsw) {
  uint32_t d;
  if constexpr (H == 0)
    asm("{\n\t.reg .b16 x1, x2, c, s, ns, z;\n\t.reg .f32 t, u, o1, o2;\n\t"
        "mov.b32 {x1, x2}, %1;\n\tmov.b32 {c, z}, %2;\n\tmov.b32 {s, z}, %3;\n\tmov.b32 {ns, z}, %4;\n\t"
        "fma.rn.f32.bf16 t, x2, ns, 0f80000000;\n\tfma.rn.f32.bf16 o1, x1, c, t;\n\t"
        "fma.rn.f32.bf16 u, x1, s, 0f80000000;\n\tfma.rn.f32.bf16 o2, x2, c, u;\n\t"
        "cvt.rn.bf16x2.f32 %0, o2, o1;\n\t}"
        : "=r"(d)
        : "r"(w), "r"(cw), "r"(sw), "r"(nsw));
  else
    asm("{\n\t.reg .b16 x1, x2, c, s, ns, z;\n\t.reg .f32 t, u, o1, o2;\n\t"
        "mov.b32 {x1, x2}, %1;\n\tmov.b32 {z, c}, %2;\n\tmov.b32 {z, s}, %3;\n\tmov.b32 {z, ns}, %4;\n\t"
        "fma.rn.f32.bf16 t, x2, ns, 0f80000000;\n\tfma.rn.f32.bf16 o1, x1, c, t;\n\t"
        "fma.rn.f32.bf16 u, x1, s, 0f80000000;\n\tfma.rn.f32.bf16 o2, x2, c, u;\n\t"
        "cvt.rn.bf16x2.f32 %0, o2, o1;\n\t}"
        : "=r"(d)
        : "r"(w), "r"(cw), "r"(sw), "r"(nsw));
  return d;
}

// A row of q_b's output after the W_UK absorb (glm_glue.cu:301-351), by ONE warp:
//  - q_pe rope into the tail of each head of qmla [T, 64, 576]: lane l owns pairs 4q .. 4q + 3
//    (q = l & 7) of heads 4k + (l >> 3), k = 0..15, so every load and store is 16 bytes and a warp
//    instruction covers four heads;
//  - on indexer layers, the indexer query: lane l holds dims 4l .. 4l + 3 of each of the 32 heads
//    (the reference's layout), rope on dims 0..63, e4m3 of v / sc with the head's UE8M0 scale (eps
//    1e-4), and the head weight ((iw * sc) * 128^-0.5) * 32^-0.5. Heads go eight at a time: one
//    reduce-scatter leaves head (l >> 2) & 7's max in lane l, which derives that head's scale.
// Every rope product is bf16 x bf16, exact in f32, so the rounding is the reference's whatever the
// contraction. sc is a power of two, so v * (1 / sc) rounds exactly as v / sc. All of the row's
// q_pe loads and the first eight heads of the query are in flight before any arithmetic.
template <bool INDEXER>
__device__ __forceinline__ void q_post_row(const bf16* __restrict__ qb, int ldb, const bf16* __restrict__ rope, int p,
                                           bf16* __restrict__ qmla, u8* __restrict__ iq, const bf16* __restrict__ iw,
                                           float* __restrict__ wout, int r, int l) {
  const u8* row = reinterpret_cast<const u8*>(qb + (size_t)r * ldb);
  const unsigned* cs = reinterpret_cast<const unsigned*>(rope + (size_t)p * 2 * HALF);
  const int q = l & 7;
  uint4 v[16];  // q_pe: pairs 4q .. 4q + 3 of heads 4k + (l >> 3)
#pragma unroll
  for (int k = 0; k < 16; ++k) v[k] = ld_stream_v4u(row + 2 * ((4 * k + (l >> 3)) * QHD + NOPE) + 16 * q);
  uint2 g0[8];  // the indexer query's heads 0..7, dims 4l .. 4l + 3
  if constexpr (INDEXER) {
#pragma unroll
    for (int k = 0; k < 8; ++k) g0[k] = ld_stream_v2(row + 2 * (HEADS * QHD + k * ID + 4 * l));
  }
  // rope values of this lane's pairs 4q .. 4q + 3: cos at cs[4q ..], sin at cs[32 + 4q ..]
  const uint2 cw = __ldg(reinterpret_cast<const uint2*>(cs) + q), sw = __ldg(reinterpret_cast<const uint2*>(cs + 16) + q);
  const uint2 nsw = make_uint2(sw.x ^ 0x80008000u, sw.y ^ 0x80008000u);
  u8* out = reinterpret_cast<u8*>(qmla + (size_t)r * HEADS * MLA);
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const int h = 4 * k + (l >> 3);
    uint4 o;
    o.x = rope_bf16<0>(v[k].x, cw.x, sw.x, nsw.x);
    o.y = rope_bf16<1>(v[k].y, cw.x, sw.x, nsw.x);
    o.z = rope_bf16<0>(v[k].z, cw.y, sw.y, nsw.y);
    o.w = rope_bf16<1>(v[k].w, cw.y, sw.y, nsw.y);
    *reinterpret_cast<uint4*>(out + 2 * (h * MLA + KVL) + 16 * q) = o;
  }
  if constexpr (INDEXER) {
    // lane l < 16 ropes dims 4l .. 4l + 3 (pairs 2l, 2l + 1)
    const unsigned c2 = l < 16 ? __ldg(cs + l) : 0u, s2 = l < 16 ? __ldg(cs + 16 + l) : 0u;
    const float ca = bf_lo(c2), sa = bf_lo(s2), cb = bf_hi(c2), sb = bf_hi(s2);
    uint2 cur[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) cur[k] = g0[k];
#pragma unroll
    for (int g = 0; g < IH / 8; ++g) {
      uint2 nxt[8];
      if (g + 1 < IH / 8) {
#pragma unroll
        for (int k = 0; k < 8; ++k) nxt[k] = ld_stream_v2(row + 2 * (HEADS * QHD + (8 * (g + 1) + k) * ID + 4 * l));
      }
      float n[8][4], m8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        n[k][0] = bf_lo(cur[k].x), n[k][1] = bf_hi(cur[k].x), n[k][2] = bf_lo(cur[k].y), n[k][3] = bf_hi(cur[k].y);
        if (l < 16) {
          const float e0 = n[k][0], o0 = n[k][1], e1 = n[k][2], o1 = n[k][3];
          n[k][0] = __fmaf_rn(e0, ca, -__fmul_rn(o0, sa));
          n[k][1] = __fmaf_rn(o0, ca, __fmul_rn(e0, sa));
          n[k][2] = __fmaf_rn(e1, cb, -__fmul_rn(o1, sb));
          n[k][3] = __fmaf_rn(o1, cb, __fmul_rn(e1, sb));
        }
        m8[k] = fmaxf(fmaxf(fabsf(n[k][0]), fabsf(n[k][1])), fmaxf(fabsf(n[k][2]), fabsf(n[k][3])));
      }
      const unsigned e = ue8m0_byte(max8_scatter(m8, l), 1e-4f);  // lane l: head 8g + ((l >> 2) & 7)
      const float inv = ue8m0_inv(e);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float iv = __shfl_sync(FULL, inv, 4 * k);
        *reinterpret_cast<uint32_t*>(iq + ((size_t)r * IH + 8 * g + k) * ID + 4 * l) =
            fp8x4(__fmul_rn(n[k][0], iv), __fmul_rn(n[k][1], iv), __fmul_rn(n[k][2], iv), __fmul_rn(n[k][3], iv));
      }
      if ((l & 3) == 0) {  // lane 4k: head 8g + k's weight
        const int ih = 8 * g + (l >> 2);
        float x = __bfloat162float(iw[(size_t)r * IH + ih]);
        x = __fmul_rn(x, __uint_as_float(e << 23));
        x = __fmul_rn(x, 0.08838834764831845f);
        x = __fmul_rn(x, 0.17677669529663687f);
        wout[(size_t)r * IH + ih] = x;
      }
      if (g + 1 < IH / 8) {
#pragma unroll
        for (int k = 0; k < 8; ++k) cur[k] = nxt[k];
      }
    }
  }
}

}  // namespace glmkv

// The rope of q_pe into qmla's tail and, when `full`, the indexer query and its head weights
// (glm_glue.cu:301-351). qb [T, ldb] bf16: 64 heads of nope 192 | pe 64, then 32 indexer heads of 128
// at column 16384. On a shared layer iq, iw and wout are null (gen.py:120-123).
//   grid ceil(T / 8), block 256: a warp a row
extern "C" __global__ void __launch_bounds__(glmkv::QP_THREADS, 2)
    glm_q_post(const glmkv::bf16* __restrict__ qb, int ldb, const glmkv::bf16* __restrict__ rope,
               const int* __restrict__ pos, glmkv::bf16* __restrict__ qmla, glmkv::u8* __restrict__ iq,
               const glmkv::bf16* __restrict__ iw, float* __restrict__ wout, int full, int T) {
  using namespace glmkv;
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x * QP_WARPS + (threadIdx.x >> 5);
  if (r >= T) return;
  if (full)
    q_post_row<true>(qb, ldb, rope, pos[r], qmla, iq, iw, wout, r, threadIdx.x & 31);
  else
    q_post_row<false>(qb, ldb, rope, pos[r], qmla, iq, iw, wout, r, threadIdx.x & 31);
}

// ================================================================================================ norm + quant glue

namespace glmkv {

constexpr int HID = 6144;                 // the residual stream's width
constexpr int ARQ_THREADS = 256;          // the reference's thread (w, l) layout, kept for its sums
constexpr int ARQ_ROW = HID * 2;          // 12288 B
constexpr int ARQ_STAGES = 2;
constexpr int ARQ_SMEM = ARQ_STAGES * 2 * ARQ_ROW;  // res and a rows of each stage: 49,152 B for two
constexpr int QT_THREADS = 256;

// max(|.|) of the eight bf16 values in a uint4, as f32
__device__ __forceinline__ float absmax8_bf16(uint4 v) {
  return absmax_bf16x2(absmax2_bf16x2(absmax2_bf16x2(v.x, v.y), absmax2_bf16x2(v.z, v.w)));
}

}  // namespace glmkv

// res = bf16(a + res) (a null: res is already the stream), written back; normed = bf16(bf16(res * rr)
// * gamma) with rr = rsqrt(block_sum(res^2) / 6144 + 1e-5); normed quantized per 128 columns into q /
// sf when q is given (glm_glue.cu:127-162). normed, q, sf may be null (gen.py:156-171).
// A persistent CTA of 256 threads takes rows b, b + G, ...: thread (w, l) holds the reference's
// columns (6w + i) * 128 + 4l + j, so the sum is built in its order. The next row's res (and a) are
// bulk-copied (TMA) into the CTA's other stage while this row is worked on.
//   persistent: grid = SMs x resident CTAs, block 256, dynamic smem ARQ_SMEM (49,152 B)
extern "C" __global__ void __launch_bounds__(glmkv::ARQ_THREADS, 3)
    glm_add_rms_quant(const glmkv::bf16* __restrict__ a, glmkv::bf16* __restrict__ res,
                      const glmkv::bf16* __restrict__ gamma, glmkv::bf16* __restrict__ normed,
                      glmkv::u8* __restrict__ q, glmkv::u8* __restrict__ sf, int sf_rows, int T) {
  using namespace glmkv;
  extern __shared__ __align__(128) u8 smem[];
  __shared__ __align__(8) unsigned long long full[ARQ_STAGES];
  __shared__ float sm[8];
  const int tid = threadIdx.x, w = tid >> 5, l = tid & 31;
  if (tid == 0) {
#pragma unroll
    for (int st = 0; st < ARQ_STAGES; ++st) mbar_init(smem_u32(&full[st]), 1);
    mbar_init_fence();
  }
  pdl_trigger();  // a persistent grid: all of its CTAs are resident
  pdl_wait();
  __syncthreads();
  int r = blockIdx.x;
  if (r >= T) return;
  const bool has_a = a != nullptr;
  const uint32_t bytes = has_a ? 2 * ARQ_ROW : ARQ_ROW;
  auto issue = [&](int st, int row) {
    const uint32_t bar = smem_u32(&full[st]);
    u8* dst = smem + (size_t)st * 2 * ARQ_ROW;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_arrive_expect_tx(bar, bytes);
    tma_load_1d(smem_u32(dst), res + (size_t)row * HID, ARQ_ROW, bar);
    if (has_a) tma_load_1d(smem_u32(dst + ARQ_ROW), a + (size_t)row * HID, ARQ_ROW, bar);
  };
  uint2 gw[6];  // gamma of this thread's columns
#pragma unroll
  for (int i = 0; i < 6; ++i) gw[i] = __ldg(reinterpret_cast<const uint2*>(gamma + (w * 6 + i) * 128 + l * 4));
  // rows r, r + G, ..., the next ARQ_STAGES - 1 of them always on their way (G = the grid)
  const long long G = gridDim.x;
  if (tid == 0)
    for (int j = 0; j < ARQ_STAGES - 1; ++j)
      if (r + j * G < T) issue(j, (int)(r + j * G));
  for (int k = 0; r < T; ++k, r += gridDim.x) {
    const int st = k % ARQ_STAGES;
    const long long rn = r + (ARQ_STAGES - 1) * G;
    // that stage held row k - 1, whose reads all came before the block_sum barriers of its iteration
    if (rn < T && tid == 0) issue((k + ARQ_STAGES - 1) % ARQ_STAGES, (int)rn);
    const bool ok = mbar_wait_bounded(smem_u32(&full[st]), (uint32_t)((k / ARQ_STAGES) & 1), WAIT_LIMIT_NS);
    if (__syncthreads_or(!ok)) {
      if (tid == 0) {  // flag it, and wait (bounded) for the copies in flight
        atomicOr(&g_fault, FAULT_WAIT_TIMEOUT);
        for (int j = 1; j < ARQ_STAGES; ++j)
          if (r + j * G < T)
            mbar_wait_bounded(smem_u32(&full[(k + j) % ARQ_STAGES]), (uint32_t)(((k + j) / ARQ_STAGES) & 1),
                              WAIT_LIMIT_NS);
      }
      return;
    }
    const u8* srow = smem + (size_t)st * 2 * ARQ_ROW;
    bf16* row = res + (size_t)r * HID;
    // v = bf16(a + res): add.rn.bf16x2 rounds the exact sum once, which equals the reference's f32
    // add then bf16 round for every pair of bf16 operands (double rounding through f32 is harmless
    // for bf16; tests/bf16_identities.cu checks all 2^32 pairs). The squares are summed in the
    // thread's column order, one mixed-precision FMA a value.
    uint2 vw[6];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 6; ++i) {
      const int c = (w * 6 + i) * 128 + l * 4;
      uint2 rv = *reinterpret_cast<const uint2*>(srow + 2 * c);
      if (has_a) {
        const uint2 av = *reinterpret_cast<const uint2*>(srow + ARQ_ROW + 2 * c);
        rv = make_uint2(add_bf16x2(rv.x, av.x), add_bf16x2(rv.y, av.y));
        *reinterpret_cast<uint2*>(row + c) = rv;
      }
      vw[i] = rv;
      ss = sq_acc4(rv, ss);
    }
    // the reference's block_sum (glm_glue.cu:57-65): warp butterflies, then the eight warp totals
    ss = warp_sum(ss);
    __syncthreads();
    if (l == 0) sm[w] = ss;
    __syncthreads();
    const float tot = warp_sum(l < 8 ? sm[l] : 0.f);
    const float rr = rsqrtf(__fadd_rn(__fdiv_rn(tot, (float)HID), EPS));
    // y = bf16(bf16(v * rr) * gamma): the first product in f32, rounded; the second is exact in f32,
    // so mul.rn.bf16x2 rounds it identically.
    const float2 rr2 = make_float2(rr, rr);
    uint2 yw[6];
#pragma unroll
    for (int i = 0; i < 6; ++i) {
      yw[i].x = mul_bf16x2(round2(mul2(unpack2(vw[i].x), rr2)), gw[i].x);
      yw[i].y = mul_bf16x2(round2(mul2(unpack2(vw[i].y), rr2)), gw[i].y);
      if (normed != nullptr) *reinterpret_cast<uint2*>(normed + (size_t)r * HID + (w * 6 + i) * 128 + l * 4) = yw[i];
    }
    if (q == nullptr) continue;
    // Per 128-column block (glm_glue.cu:86-92): the warp's six blocks' |max| in three packed words
    // (blocks 2j | 2j + 1), reduced and scattered so lane l holds block 2 ((l >> 3) & 3) + (l & 1)
    // (lanes 24..31 hold padding); UE8M0 scale (eps 1e-10) there, then e4m3 of y * (1 / scale).
    uint32_t m2[4];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const uint32_t x0 = absmax_xs(yw[2 * j].x, yw[2 * j].y), x1 = absmax_xs(yw[2 * j + 1].x, yw[2 * j + 1].y);
      m2[j] = absmax_xs(__byte_perm(x0, x1, 0x5410), __byte_perm(x0, x1, 0x7632));
    }
    m2[3] = 0u;
    const bool b4 = l & 16, b3 = l & 8;
    const uint32_t a0 = absmax_xs(b4 ? m2[2] : m2[0], __shfl_xor_sync(FULL, b4 ? m2[0] : m2[2], 16));
    const uint32_t a1 = absmax_xs(b4 ? m2[3] : m2[1], __shfl_xor_sync(FULL, b4 ? m2[1] : m2[3], 16));
    uint32_t mw = absmax_xs(b3 ? a1 : a0, __shfl_xor_sync(FULL, b3 ? a0 : a1, 8));
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) mw = absmax_xs(mw, __shfl_xor_sync(FULL, mw, o));
    const float bm = __uint_as_float(((l & 1) ? (mw & 0xffff0000u) : (mw << 16)) & 0x7fffffffu);
    const unsigned e = ue8m0_byte(bm, 1e-10f);
    const uint32_t inv = __float_as_uint(ue8m0_inv(e));
    u8* qrow = q + (size_t)r * HID;
#pragma unroll
    for (int i = 0; i < 6; ++i) {
      const uint32_t iv = __shfl_sync(FULL, inv, 8 * (i >> 1) + (i & 1));
      const float2 p0 = scale_bf16x2(yw[i].x, iv), p1 = scale_bf16x2(yw[i].y, iv);
      *reinterpret_cast<uint32_t*>(qrow + (w * 6 + i) * 128 + l * 4) = fp8x4(p0.x, p0.y, p1.x, p1.y);
    }
    const int bk = 2 * ((l >> 3) & 3) + (l & 1), kb = w * 6 + bk;
    if ((l & 6) == 0 && bk < 6) sf[((size_t)(kb >> 2) * sf_rows + r) * 4 + (kb & 3)] = (u8)e;
  }
}

// x [T, K] bf16 (rows ldx apart) quantized per 128 columns into q [T, K] e4m3 and DeepGEMM's packed
// UE8M0 words [(K / 512)][sf_rows] (glm_glue.cu:164-175). A warp takes four consecutive blocks of a
// row; lane l holds 16 values of block l >> 3 (two 16-byte loads), the block's amax is three
// shuffles, and lane 0 writes the four scale bytes as one word.
//   grid ceil(T * ceil(K / 512) / 8), block 256
extern "C" __global__ void __launch_bounds__(glmkv::QT_THREADS)
    glm_quant(const glmkv::bf16* __restrict__ x, int ldx, glmkv::u8* __restrict__ q, glmkv::u8* __restrict__ sf,
              int sf_rows, int K, int T) {
  using namespace glmkv;
  pdl_trigger();
  pdl_wait();
  const int nb = K >> 7, ng = (nb + 3) >> 2;
  const long long gwarp = ((long long)blockIdx.x * QT_THREADS + threadIdx.x) >> 5;
  if (gwarp >= (long long)T * ng) return;
  const int r = (int)(gwarp / ng), m = (int)(gwarp % ng), l = threadIdx.x & 31;
  const int kb = 4 * m + (l >> 3);
  const bool live = kb < nb;
  const int col = kb * 128 + 16 * (l & 7);
  uint4 v0 = make_uint4(0, 0, 0, 0), v1 = v0;
  if (live) {
    const u8* src = reinterpret_cast<const u8*>(x + (size_t)r * ldx + col);
    v0 = ld_stream_v4u(src);
    v1 = ld_stream_v4u(src + 16);
  }
  float amax = fmaxf(absmax8_bf16(v0), absmax8_bf16(v1));
  amax = fmaxf(amax, __shfl_xor_sync(FULL, amax, 4));
  amax = fmaxf(amax, __shfl_xor_sync(FULL, amax, 2));
  amax = fmaxf(amax, __shfl_xor_sync(FULL, amax, 1));
  const unsigned e = ue8m0_byte(amax, 1e-10f);
  const float inv = ue8m0_inv(e);
  const float2 i2 = make_float2(inv, inv);
  const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 p0 = mul2(unpack2(w[2 * i]), i2), p1 = mul2(unpack2(w[2 * i + 1]), i2);
    o[i] = fp8x4(p0.x, p0.y, p1.x, p1.y);
  }
  if (live) *reinterpret_cast<uint4*>(q + (size_t)r * K + col) = make_uint4(o[0], o[1], o[2], o[3]);
  const unsigned e1 = __shfl_sync(FULL, e, 8), e2 = __shfl_sync(FULL, e, 16), e3 = __shfl_sync(FULL, e, 24);
  if (l == 0) {
    u8* word = sf + ((size_t)m * sf_rows + r) * 4;
    if (4 * m + 3 < nb) {
      *reinterpret_cast<unsigned*>(word) = e | (e1 << 8) | (e2 << 16) | (e3 << 24);
    } else {  // the row's last blocks: byte stores for the ones that exist
      word[0] = (u8)e;
      if (4 * m + 1 < nb) word[1] = (u8)e1;
      if (4 * m + 2 < nb) word[2] = (u8)e2;
    }
  }
}

// Self-test of the bounded wait every pipeline uses: one thread waits on an mbarrier that nothing
// ever arrives on, gives up after `limit_ns`, sets FAULT_WAIT_TIMEOUT and returns. No counterpart
// in the reference.
//   grid 1, block 32
extern "C" __global__ void glmkv_wait_selftest_kernel(unsigned long long limit_ns, unsigned* __restrict__ waited_ns) {
  using namespace glmkv;
  __shared__ __align__(8) unsigned long long bar;
  if (threadIdx.x != 0) return;
  mbar_init(smem_u32(&bar), 1);
  mbar_init_fence();
  const uint64_t t0 = global_ns();
  if (!mbar_wait_bounded(smem_u32(&bar), 0u, limit_ns)) atomicOr(&g_fault, FAULT_WAIT_TIMEOUT);
  const uint64_t dt = global_ns() - t0;
  *waited_ns = dt > 0xffffffffull ? 0xffffffffu : (unsigned)dt;
}
