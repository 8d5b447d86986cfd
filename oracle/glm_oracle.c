/*
 * CPU oracle for the KV-cache path of kern-glm53's glue kernels.
 *
 * TEST INFRASTRUCTURE ONLY. This file restates, in plain C, what the reference kernels in
 * kern-glm53 `source/glm_glue.cu` compute, so that the CUDA kernels of this repository can be
 * checked against it. Only `tests/`, `__graft_entry__.smoke()` and the `cpu_baseline` leg of
 * `bench.py` may load it. Nothing in the product path calls it.
 *
 * Every function cites the reference lines it follows. The arithmetic is spelled out step by step
 * (this file is compiled with -ffp-contract=off): every f32 rounding the GPU performs is a separate
 * C float operation here, and the fused multiply-adds the reference's compiled code performs are
 * explicit fmaf() calls. Reductions reproduce the reference's exact association order (per-thread
 * sequential partials, the 32-lane xor butterfly, then the butterfly over the block's eight warp
 * totals).
 *
 * The one step that is not restated bit for bit is CUDA's rsqrtf (an approximate hardware
 * reciprocal square root). The oracle uses the correctly rounded 1/sqrt instead, so rows whose
 * RMS / LayerNorm factor lands on a different f32 may differ by one bf16 ulp / one e4m3 code.
 * Tests compare those outputs with that tolerance; the bit-exact verdict on them comes from the
 * reference kernels themselves, compiled from source and run on the GPU.
 *
 * Conversions follow their published definitions:
 *   bf16: the top 16 bits of an IEEE f32, rounded to nearest even (NaN -> 0x7FFF).
 *   e4m3 (OCP FP8 E4M3FN): bias 7, no infinities, 0x7F/0xFF NaN, max finite 448; "satfinite"
 *   conversion rounds to nearest even and clamps finite overflow to +-448.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define QL 2048
#define KVL 512
#define HALF 32
#define MLA 576
#define ID 128
#define TOPK 2048
#define PAGE 64
#define IDX_PAGE (PAGE * (ID + 4))
#define KV8 (KVL + 16 + 2 * 64)
#define EPS 1e-5f

/* ---------------------------------------------------------------- scalar formats */

static inline float f_of(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t u_of(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

static inline float bf16_f(uint16_t h) { return f_of((uint32_t)h << 16); }

/* f32 -> bf16, round to nearest even (glm_glue.cu:43 `rnd`, __float2bfloat16). */
static inline uint16_t f_bf16(float f) {
  uint32_t u = u_of(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fff;
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
static inline float rnd(float f) { return bf16_f(f_bf16(f)); }

/* f32 -> e4m3 with satfinite, round to nearest even (glm_glue.cu:76-79, 245-246). */
static inline uint8_t f_e4m3(float f) {
  uint32_t u = u_of(f);
  uint8_t s = (uint8_t)((u >> 24) & 0x80u);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7f;
  float a = fabsf(f);
  if (a >= 448.0f) return s | 0x7e;
  if (a < 0.015625f) {                       /* below 2^-6: subnormal grid of 2^-9 */
    float m = nearbyintf(a * 512.0f);        /* exact scaling, RNE to an integer 0..8 */
    return s | (uint8_t)m;
  }
  int e;
  frexpf(a, &e);                             /* a = f * 2^e, f in [0.5, 1): exponent e-1 */
  e -= 1;                                    /* -6 .. 8 */
  float m = nearbyintf(ldexpf(a, 3 - e));    /* 8 .. 16 */
  return s | (uint8_t)((e + 6) * 8 + (int)m);
}

/* e4m3 -> f32, exact (glm_glue.cu:405-407). */
static inline float e4m3_f(uint8_t b) {
  int e = (b >> 3) & 15, m = b & 7;
  if (e == 15 && m == 7) return NAN;
  float v = e == 0 ? ldexpf((float)m, -9) : ldexpf((float)(8 + m), e - 10);
  return (b & 0x80) ? -v : v;
}

/* The UE8M0 scale (glm_glue.cu:68-74). */
static inline float ue8m0(float amax, float eps, uint8_t* e) {
  const uint32_t b = u_of(fmaxf(amax, eps) / 448.0f);
  uint32_t x = (b >> 23) & 0xffu;
  x += (b & 0x7fffffu) != 0;
  *e = (uint8_t)x;
  return f_of(x << 23);
}

/* Correctly rounded 1/sqrt: stands in for CUDA's rsqrtf (see the header). */
static inline float rsqrt_cr(float x) { return (float)(1.0 / sqrt((double)x)); }

/* ---------------------------------------------------------------- reductions */

/* `warp_sum` (glm_glue.cu:45-49): v += shfl_xor(v, o) for o = 16 .. 1; every lane ends equal. */
static float warp_sum32(const float* v) {
  float a[32], b[32];
  memcpy(a, v, sizeof a);
  for (int o = 16; o; o >>= 1) {
    for (int l = 0; l < 32; ++l) b[l] = a[l] + a[l ^ o];
    memcpy(a, b, sizeof a);
  }
  return a[0];
}

/* `block_sum` over 8 warps (glm_glue.cu:57-65): warp totals, then warp_sum of {S0..S7, 0 x 24}. */
static float block_sum256(const float* v) {
  float t[32] = {0};
  for (int w = 0; w < 8; ++w) t[w] = warp_sum32(v + 32 * w);
  return warp_sum32(t);
}

/* ---------------------------------------------------------------- glm_plan */

/* glm_glue.cu:109-125 */
void orc_plan(const int64_t* cu, const int32_t* seq_lens, int nseq, int32_t* pos, uint32_t* ks, uint32_t* ke,
              int32_t* klen, int32_t* row_seq, int32_t* zero, int T) {
  for (int r = 0; r < T; ++r) {
    int s = 0;
    uint32_t goff = 0;
    while (s + 1 < nseq && cu[s + 1] <= r) goff += (uint32_t)seq_lens[s++];
    const int p = seq_lens[s] - (int)(cu[s + 1] - r);
    pos[r] = p;
    ks[r] = goff;
    ke[r] = goff + (uint32_t)p + 1u;
    klen[r] = p + 1;
    row_seq[r] = s;
    zero[r] = 0;
  }
}

/* ---------------------------------------------------------------- glm_mla_prep{,_fp8} */

/* Contraction pattern of the indexer-key arithmetic (glm_glue.cu:263-279) as the reference's
 * compiled code (nvcc 12.9, sm_100a, -O3) evaluates it, found by running the reference kernel on
 * 2^20 rows against every combination: only this one matches all of them. Bit 0: d2 += d*d fused;
 * bit 1: n = (d*rstd)*w + b with the last multiply fused; bit 2: the rope as fma(e, c, -(o*sn))
 * and fma(e, sn, o*c). A cleared bit evaluates that step with separate roundings. */
static int g_idx_fma = 7;
void orc_set_idx_fma(int flags) { g_idx_fma = flags; }
int orc_get_idx_fma(void) { return g_idx_fma; }

/* One row of mla_prep (glm_glue.cu:202-287). x is bf16 bits. kv / idx may be NULL-skipped as in
 * the reference: slot < 0 skips every cache write, idx == NULL skips the indexer key. */
static void prep_row(int fp8, const uint16_t* x, int lda, const uint16_t* g_q, const uint16_t* g_kv,
                     const uint16_t* rope, const int32_t* pos, const int64_t* slot, uint8_t* kv, uint8_t* idx,
                     const uint16_t* ik_w, const uint16_t* ik_b, uint8_t* qq, uint8_t* qsf, int sf_rows, int r) {
  const uint16_t* row = x + (size_t)r * lda;
  float part[256];
  /* q_a: thread t (warp w, lane l) holds columns (2w + i) * 128 + 4l + j (glm_glue.cu:212-217). */
  for (int t = 0; t < 256; ++t) {
    const int w = t >> 5, l = t & 31;
    float ss = 0.f;
    for (int i = 0; i < 2; ++i)
      for (int j = 0; j < 4; ++j) {
        const float v = bf16_f(row[(w * 2 + i) * 128 + l * 4 + j]);
        ss = ss + v * v; /* the square of a bf16 value is exact in f32 */
      }
    part[t] = ss;
  }
  const float rq = rsqrt_cr(block_sum256(part) / (float)QL + EPS);
  /* kv_a: thread t holds columns 2t, 2t+1 (glm_glue.cu:218-219) */
  for (int t = 0; t < 256; ++t) {
    const float a = bf16_f(row[QL + 2 * t]), b = bf16_f(row[QL + 2 * t + 1]);
    part[t] = a * a + b * b;
  }
  const float rk = rsqrt_cr(block_sum256(part) / (float)KVL + EPS);

  /* q_c quantized per 128 columns into qq / qsf (glm_glue.cu:222-230, 86-92, 81-83) */
  for (int kb = 0; kb < QL / 128; ++kb) {
    float y[128], amax = 0.f;
    for (int c = 0; c < 128; ++c) {
      const int col = kb * 128 + c;
      float t = bf16_f(row[col]) * rq;
      t = t * bf16_f(g_q[col]);
      y[c] = rnd(t);
      amax = fmaxf(amax, fabsf(y[c]));
    }
    uint8_t e;
    const float inv = 1.0f / ue8m0(amax, 1e-10f, &e);
    for (int c = 0; c < 128; ++c) qq[(size_t)r * QL + kb * 128 + c] = f_e4m3(y[c] * inv);
    qsf[((size_t)(kb >> 2) * sf_rows + r) * 4 + (kb & 3)] = e;
  }

  const int64_t s = slot[r];
  if (s < 0) return;
  const int p = pos[r];
  const uint16_t* cs = rope + (size_t)p * 2 * HALF;
  uint8_t* dst = kv + s * (fp8 ? KV8 : MLA * 2);
  float k[512];
  for (int c = 0; c < 512; ++c) {
    float t = bf16_f(row[QL + c]) * rk;
    t = t * bf16_f(g_kv[c]);
    k[c] = rnd(t);
  }
  if (fp8) {
    /* four tiles of 128, scale amax / 448 (glm_glue.cu:238-247) */
    for (int tile = 0; tile < 4; ++tile) {
      float m = 0.f;
      for (int c = 0; c < 128; ++c) m = fmaxf(m, fabsf(k[tile * 128 + c]));
      const float sc = m / 448.0f, inv = sc > 0.f ? 1.0f / sc : 0.f;
      for (int c = 0; c < 128; ++c) dst[tile * 128 + c] = f_e4m3(k[tile * 128 + c] * inv);
      memcpy(dst + KVL + 4 * tile, &sc, 4);
    }
  } else {
    for (int c = 0; c < 512; ++c) {
      const uint16_t h = f_bf16(k[c]);
      memcpy(dst + 2 * c, &h, 2);
    }
  }
  /* k_pe rope, interleaved pairs (glm_glue.cu:252-257); bf16 products are exact in f32 */
  uint8_t* pe = dst + (fp8 ? KVL + 16 : KVL * 2);
  for (int t = 0; t < HALF; ++t) {
    const float x1 = bf16_f(row[QL + KVL + 2 * t]), x2 = bf16_f(row[QL + KVL + 2 * t + 1]);
    const float c = bf16_f(cs[t]), sn = bf16_f(cs[HALF + t]);
    const uint16_t a = f_bf16(x1 * c - x2 * sn), b = f_bf16(x2 * c + x1 * sn);
    memcpy(pe + 4 * t, &a, 2);
    memcpy(pe + 4 * t + 2, &b, 2);
  }
  if (idx == NULL) return;

  /* indexer key: LayerNorm, rope on dims 0..63, UE8M0 e4m3 (glm_glue.cu:258-286), one warp */
  float kk[32][4], kw[32][4], kbias[32][4], lanes[32];
  for (int l = 0; l < 32; ++l)
    for (int j = 0; j < 4; ++j) {
      kk[l][j] = bf16_f(row[QL + KVL + 2 * HALF + l * 4 + j]);
      kw[l][j] = bf16_f(ik_w[l * 4 + j]);
      kbias[l][j] = bf16_f(ik_b[l * 4 + j]);
    }
  for (int l = 0; l < 32; ++l) lanes[l] = ((kk[l][0] + kk[l][1]) + kk[l][2]) + kk[l][3];
  const float mean = warp_sum32(lanes) / (float)ID;
  for (int l = 0; l < 32; ++l) {
    float d2 = 0.f;
    for (int j = 0; j < 4; ++j) {
      const float d = kk[l][j] - mean;
      d2 = (g_idx_fma & 1) ? fmaf(d, d, d2) : d2 + d * d;
    }
    lanes[l] = d2;
  }
  const float rstd = rsqrt_cr(warp_sum32(lanes) / (float)ID + 1e-6f);
  float n[32][4], amax = 0.f;
  for (int l = 0; l < 32; ++l) {
    for (int j = 0; j < 4; ++j) {
      const float t = (kk[l][j] - mean) * rstd;
      n[l][j] = (g_idx_fma & 2) ? fmaf(t, kw[l][j], kbias[l][j]) : t * kw[l][j] + kbias[l][j];
    }
    if (l < 16) {
      for (int j = 0; j < 4; j += 2) {
        const int pr = (l * 4 + j) >> 1;
        const float c = bf16_f(cs[pr]), sn = bf16_f(cs[HALF + pr]), e = n[l][j], o = n[l][j + 1];
        if (g_idx_fma & 4) {
          n[l][j] = fmaf(e, c, -(o * sn));
          n[l][j + 1] = fmaf(e, sn, o * c);
        } else {
          n[l][j] = e * c - o * sn;
          n[l][j + 1] = o * c + e * sn;
        }
      }
    }
    for (int j = 0; j < 4; ++j) amax = fmaxf(amax, fabsf(n[l][j]));
  }
  uint8_t e;
  const float sc = ue8m0(amax, 1e-4f, &e);
  uint8_t* page = idx + (size_t)(s / PAGE) * IDX_PAGE;
  const int i = (int)(s % PAGE);
  for (int l = 0; l < 32; ++l)
    for (int j = 0; j < 4; ++j) page[i * ID + l * 4 + j] = f_e4m3(n[l][j] / sc);
  memcpy(page + PAGE * ID + 4 * i, &sc, 4);
}

/* glm_glue.cu:294-299. Rows are independent except for their cache slots (unique per token). */
void orc_mla_prep(int fp8, const uint16_t* x, int lda, const uint16_t* g_q, const uint16_t* g_kv,
                  const uint16_t* rope, const int32_t* pos, const int64_t* slot, uint8_t* kv, uint8_t* idx,
                  const uint16_t* ik_w, const uint16_t* ik_b, uint8_t* qq, uint8_t* qsf, int sf_rows, int T) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < T; ++r)
    prep_row(fp8, x, lda, g_q, g_kv, rope, pos, slot, kv, idx, ik_w, ik_b, qq, qsf, sf_rows, r);
}

/* ---------------------------------------------------------------- paged reads */

/* The pages of every sequence in order: page j of sequence s covers rows [64j, min(64j+64, len))
 * and lands at stream rows goff(s) + 64j (glm_glue.cu:360-371, 385-395). */
typedef struct { int s, j, n; uint64_t row; } page_ref;

static long count_pages(const int32_t* seq_lens, int nseq) {
  long np = 0;
  for (int s = 0; s < nseq; ++s) np += (seq_lens[s] + PAGE - 1) / PAGE;
  return np;
}

static page_ref page_at(const int32_t* seq_lens, int nseq, long b) {
  page_ref pr = {nseq, 0, 0, 0};
  uint32_t goff = 0; /* the reference's stream offset is an unsigned 32-bit sum */
  for (int s = 0; s < nseq; ++s) {
    const long pages = (seq_lens[s] + PAGE - 1) / PAGE;
    if (b < pages) {
      pr.s = s;
      pr.j = (int)b;
      pr.n = seq_lens[s] - (int)b * PAGE < PAGE ? seq_lens[s] - (int)b * PAGE : PAGE;
      pr.row = (uint64_t)goff + (uint64_t)b * PAGE;
      return pr;
    }
    b -= pages;
    goff += (uint32_t)seq_lens[s];
  }
  return pr;
}

/* glm_idx_gather, glm_glue.cu:357-376 */
void orc_idx_gather(const uint8_t* idx, const int32_t* block_table, int max_pages, const int32_t* seq_lens, int nseq,
                    uint8_t* kg, float* ksf) {
  const long np = count_pages(seq_lens, nseq);
#pragma omp parallel for schedule(static)
  for (long b = 0; b < np; ++b) {
    const page_ref pr = page_at(seq_lens, nseq, b);
    const uint8_t* src = idx + (size_t)block_table[(size_t)pr.s * max_pages + pr.j] * IDX_PAGE;
    memcpy(kg + pr.row * ID, src, (size_t)pr.n * ID);
    memcpy(ksf + pr.row, src + PAGE * ID, (size_t)pr.n * 4);
  }
}

/* glm_kv_dequant, glm_glue.cu:382-414: bf16(f32(e4m3) * tile scale), k_pe copied verbatim. */
void orc_kv_dequant(const uint8_t* kv, const int32_t* block_table, int max_pages, const int32_t* seq_lens, int nseq,
                    uint16_t* kvd) {
  float lut[256];
  for (int b = 0; b < 256; ++b) lut[b] = e4m3_f((uint8_t)b);
  const long np = count_pages(seq_lens, nseq);
#pragma omp parallel for schedule(static)
  for (long b = 0; b < np; ++b) {
    const page_ref pr = page_at(seq_lens, nseq, b);
    const uint8_t* page = kv + (size_t)block_table[(size_t)pr.s * max_pages + pr.j] * PAGE * KV8;
    for (int i = 0; i < pr.n; ++i) {
      const uint8_t* src = page + (size_t)i * KV8;
      uint16_t* dst = kvd + (pr.row + i) * MLA;
      for (int tile = 0; tile < 4; ++tile) {
        float sc;
        memcpy(&sc, src + KVL + 4 * tile, 4);
        for (int c = 0; c < 128; ++c) dst[tile * 128 + c] = f_bf16(lut[src[tile * 128 + c]] * sc);
      }
      memcpy(dst + KVL, src + KVL + 16, 128);
    }
  }
}

/* ---------------------------------------------------------------- row plans */

/* glm_topk_stream, glm_glue.cu:419-428 */
void orc_topk_stream(int32_t* ind, const uint32_t* ks, const int32_t* klen, int32_t* tlen, int T) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < T; ++r) {
    int32_t* row = ind + (size_t)r * TOPK;
    for (int i = 0; i < TOPK; ++i) {
      const int32_t k = row[i];
      row[i] = k < 0 ? -1 : (int32_t)(ks[r] + (uint32_t)k);
    }
    tlen[r] = klen[r] < TOPK ? klen[r] : TOPK;
  }
}

/* glm_topk_slots, glm_glue.cu:433-444 */
void orc_topk_slots(int32_t* ind, const int32_t* block_table, int max_pages, const int32_t* row_seq,
                    const int32_t* klen, int32_t* tlen, int T) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < T; ++r) {
    const int32_t* bt = block_table + (size_t)row_seq[r] * max_pages;
    int32_t* row = ind + (size_t)r * TOPK;
    for (int i = 0; i < TOPK; ++i) {
      const int32_t k = row[i];
      row[i] = k < 0 ? -1 : bt[k / PAGE] * PAGE + k % PAGE;
    }
    tlen[r] = klen[r] < TOPK ? klen[r] : TOPK;
  }
}

/* ---------------------------------------------------------------- glm_q_post */

#define HEADS 64
#define QHD 256
#define NOPE 192
#define IH 32

/* glm_glue.cu:301-351: the q_pe rope into the tail of each head of qmla [T, 64, 576], and on full
 * layers the indexer query: rope on its first 64 dims, e4m3 per (row, head) with a UE8M0 scale
 * (eps 1e-4), and the head weight w = ((f32(iw) * sc) * 128^-0.5) * 32^-0.5. Every rope product is
 * bf16 x bf16, exact in f32, so no contraction can change a bit. */
void orc_q_post(const uint16_t* qb, int ldb, const uint16_t* rope, const int32_t* pos, uint16_t* qmla, uint8_t* iq,
                const uint16_t* iw, float* wout, int full, int T) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < T; ++r) {
    const uint16_t* row = qb + (size_t)r * ldb;
    const uint16_t* cs = rope + (size_t)pos[r] * 2 * HALF;
    for (int h = 0; h < HEADS; ++h)
      for (int pr = 0; pr < HALF; ++pr) {
        const float x1 = bf16_f(row[h * QHD + NOPE + 2 * pr]), x2 = bf16_f(row[h * QHD + NOPE + 2 * pr + 1]);
        const float c = bf16_f(cs[pr]), sn = bf16_f(cs[HALF + pr]);
        uint16_t* d = qmla + ((size_t)r * HEADS + h) * MLA + KVL + 2 * pr;
        d[0] = f_bf16(x1 * c - x2 * sn);
        d[1] = f_bf16(x2 * c + x1 * sn);
      }
    if (!full) continue;
    for (int ih = 0; ih < IH; ++ih) {
      float v[ID], amax = 0.f;
      for (int j = 0; j < ID; ++j) v[j] = bf16_f(row[HEADS * QHD + ih * ID + j]);
      for (int pr = 0; pr < HALF; ++pr) {
        const float c = bf16_f(cs[pr]), sn = bf16_f(cs[HALF + pr]), e = v[2 * pr], o = v[2 * pr + 1];
        v[2 * pr] = e * c - o * sn;
        v[2 * pr + 1] = o * c + e * sn;
      }
      for (int j = 0; j < ID; ++j) amax = fmaxf(amax, fabsf(v[j]));
      uint8_t e;
      const float sc = ue8m0(amax, 1e-4f, &e);
      for (int j = 0; j < ID; ++j) iq[((size_t)r * IH + ih) * ID + j] = f_e4m3(v[j] / sc);
      float x = bf16_f(iw[(size_t)r * IH + ih]);
      x *= sc;
      x *= 0.08838834764831845f;
      x *= 0.17677669529663687f;
      wout[(size_t)r * IH + ih] = x;
    }
  }
}

/* ---------------------------------------------------------------- glm_add_rms_quant, glm_quant */

#define HID 6144

/* Four values of a 128-column block quantized (glm_glue.cu:85-92): amax of the block, UE8M0 scale
 * with eps 1e-10, e4m3 of v * (1 / scale); the exponent byte into DeepGEMM's packed layout. */
static void quant_block(const float* y, uint8_t* q, uint8_t* sf, int sf_rows, int r, int kb) {
  float amax = 0.f;
  for (int c = 0; c < 128; ++c) amax = fmaxf(amax, fabsf(y[c]));
  uint8_t e;
  const float inv = 1.0f / ue8m0(amax, 1e-10f, &e);
  for (int c = 0; c < 128; ++c) q[c] = f_e4m3(y[c] * inv);
  sf[((size_t)(kb >> 2) * sf_rows + r) * 4 + (kb & 3)] = e;
}

/* glm_glue.cu:127-162: res = bf16(a + res) when a is given (written back), then
 * normed = bf16(bf16(res * rr) * gamma), rr = rsqrt(block_sum(res^2) / 6144 + 1e-5), quantized per 128
 * columns when q is given. Thread (w, l) of the reference's 256 holds columns (6w + i) * 128 + 4l + j. */
void orc_add_rms_quant(const uint16_t* a, uint16_t* res, const uint16_t* gamma, uint16_t* normed, uint8_t* q,
                       uint8_t* sf, int sf_rows, int T) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < T; ++r) {
    uint16_t* row = res + (size_t)r * HID;
    float v[HID], part[256];
    for (int c = 0; c < HID; ++c) {
      v[c] = bf16_f(row[c]);
      if (a) {
        v[c] = rnd(v[c] + bf16_f(a[(size_t)r * HID + c]));
        row[c] = f_bf16(v[c]);
      }
    }
    for (int t = 0; t < 256; ++t) {
      const int w = t >> 5, l = t & 31;
      float ss = 0.f;
      for (int i = 0; i < 6; ++i)
        for (int j = 0; j < 4; ++j) {
          const float x = v[(w * 6 + i) * 128 + l * 4 + j];
          ss = ss + x * x;
        }
      part[t] = ss;
    }
    const float rr = rsqrt_cr(block_sum256(part) / (float)HID + EPS);
    float y[HID];
    for (int c = 0; c < HID; ++c) {
      float t = v[c] * rr;
      t = rnd(t) * bf16_f(gamma[c]);
      y[c] = rnd(t);
      if (normed) normed[(size_t)r * HID + c] = f_bf16(y[c]);
    }
    if (q)
      for (int kb = 0; kb < HID / 128; ++kb) quant_block(y + kb * 128, q + (size_t)r * HID + kb * 128, sf, sf_rows, r, kb);
  }
}

/* glm_glue.cu:164-175: x [T, K] (rows ldx apart) quantized per 128 columns into q [T, K] and sf. */
void orc_quant(const uint16_t* x, int ldx, uint8_t* q, uint8_t* sf, int sf_rows, int K, int T) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < T; ++r)
    for (int kb = 0; kb < (K >> 7); ++kb) {
      float y[128];
      for (int c = 0; c < 128; ++c) y[c] = bf16_f(x[(size_t)r * ldx + kb * 128 + c]);
      quant_block(y, q + (size_t)r * K + kb * 128, sf, sf_rows, r, kb);
    }
}

/* ---------------------------------------------------------------- helpers exported for tests */

void orc_bf16_from_f32(const float* x, uint16_t* y, long n) {
  for (long i = 0; i < n; ++i) y[i] = f_bf16(x[i]);
}
void orc_e4m3_from_f32(const float* x, uint8_t* y, long n) {
  for (long i = 0; i < n; ++i) y[i] = f_e4m3(x[i]);
}
void orc_f32_from_e4m3(const uint8_t* x, float* y, long n) {
  for (long i = 0; i < n; ++i) y[i] = e4m3_f(x[i]);
}
int orc_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
void orc_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
