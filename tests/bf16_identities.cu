// The Blackwell bf16 instructions the kernels use in place of f32 arithmetic, checked against the
// f32 forms the reference computes, on this GPU. Each check counts mismatches over an input space:
//
//   add.rn.bf16x2 (a, b)              == bf16_rn(f32 a + f32 b)            all 2^32 bf16 pairs
//   mul.rn.bf16x2 (a, b)              == bf16_rn(f32 a * f32 b)            all 2^32 bf16 pairs
//   fma.rn.f32.bf16 (y, s, -0)        == f32 y * f32 s                     all 2^32 bf16 pairs
//   fma.rn.f32.bf16 (a, a, c)         == fmaf(f32 a, f32 a, c)             all bf16 a x 2^16 f32 c
//   fma.rn.f32.bf16 (a, b, c)         == fmaf(f32 a, f32 b, c)             all 2^32 bf16 pairs, c hashed
//   max.xorsign.abs.bf16x2 (a, b)     == fmaxf(|f32 a|, |f32 b|)           all 2^32 bf16 pairs
//                                        (magnitude; NaN-vs-NaN encodings counted apart)
//
// Printed as one line: name=mismatches[/nan_encoding_only] ... ; exit status 0 when all are zero.
// Built and run by tests/test_gpu_bf16_identities.py.
#include <cuda_bf16.h>

#include <cstdint>
#include <cstdio>

__device__ __forceinline__ float widen(uint32_t h) { return __uint_as_float(h << 16); }
__device__ __forceinline__ uint32_t bf16_rn(float x) {
  const __nv_bfloat16 b = __float2bfloat16_rn(x);
  return *reinterpret_cast<const uint16_t*>(&b);
}
__device__ __forceinline__ bool nan16(uint32_t h) { return (h & 0x7f80u) == 0x7f80u && (h & 0x7fu) != 0u; }

enum { ADD, MUL, SCALE, SQ, FMA, MAXABS, NCHECK };

__global__ void check_pairs(unsigned long long* bad, unsigned long long* nan_only) {
  unsigned long long b[NCHECK] = {}, n[NCHECK] = {};
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < (1ull << 32); i += stride) {
    const uint32_t a = (uint32_t)(i >> 16), c = (uint32_t)(i & 0xffffu);
    const uint32_t x = a | (c << 16), y = c | (a << 16);  // both operand orders, one in each half
    uint32_t s, m, mx;
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(s) : "r"(x), "r"(y));
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(m) : "r"(x), "r"(y));
    asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(mx) : "r"(x), "r"(y));
    const uint32_t want_s[2] = {bf16_rn(__fadd_rn(widen(a), widen(c))), bf16_rn(__fadd_rn(widen(c), widen(a)))};
    const uint32_t want_m[2] = {bf16_rn(__fmul_rn(widen(a), widen(c))), bf16_rn(__fmul_rn(widen(c), widen(a)))};
    const uint32_t want_mx = __float_as_uint(fmaxf(fabsf(widen(a)), fabsf(widen(c)))) >> 16;
    for (int h = 0; h < 2; ++h) {
      const uint32_t gs = (s >> (16 * h)) & 0xffffu, gm = (m >> (16 * h)) & 0xffffu;
      const uint32_t gx = (mx >> (16 * h)) & 0x7fffu;
      if (gs != want_s[h]) ++(nan16(gs) && nan16(want_s[h]) ? n[ADD] : b[ADD]);
      if (gm != want_m[h]) ++(nan16(gm) && nan16(want_m[h]) ? n[MUL] : b[MUL]);
      if (gx != want_mx) ++(nan16(gx) && nan16(want_mx) ? n[MAXABS] : b[MAXABS]);
    }
    float d;
    asm("{\n\t.reg .b16 p, q, z;\n\tmov.b32 {p, z}, %1;\n\tmov.b32 {q, z}, %2;\n\t"
        "fma.rn.f32.bf16 %0, p, q, 0f80000000;\n\t}"
        : "=f"(d)
        : "r"(a), "r"(c));
    const float want_d = __fmul_rn(widen(a), widen(c));
    if (__float_as_uint(d) != __float_as_uint(want_d)) ++(d != d && want_d != want_d ? n[SCALE] : b[SCALE]);
    // a^2 + acc for an f32 accumulator spread over every exponent: acc bits = c << 16 | (a * 40503) & 0xffff
    const float acc = __uint_as_float((c << 16) | ((a * 40503u) & 0xffffu));
    float e;
    asm("{\n\t.reg .b16 p, z;\n\tmov.b32 {p, z}, %1;\n\tfma.rn.f32.bf16 %0, p, p, %2;\n\t}" : "=f"(e) : "r"(a), "f"(acc));
    const float want_e = __fmaf_rn(widen(a), widen(a), acc);
    if (__float_as_uint(e) != __float_as_uint(want_e)) ++(e != e && want_e != want_e ? n[SQ] : b[SQ]);
    // a * c + an addend near the product's magnitude (exponent of a * c, +-24) or anywhere, by a hash of i
    const uint32_t hsh = (uint32_t)(i * 0x9E3779B97F4A7C15ull >> 32);
    const float pr = __fmul_rn(widen(a), widen(c));
    const uint32_t pe = (__float_as_uint(pr) >> 23) & 0xffu;
    const uint32_t ae = (hsh & 1u) ? (hsh >> 24) : (uint32_t)min(254, max(1, (int)pe + (int)((hsh >> 24) % 49u) - 24));
    const float addend = __uint_as_float((hsh & 0x80000000u) | (ae << 23) | ((hsh >> 1) & 0x7fffffu));
    float f;
    asm("{\n\t.reg .b16 p, q, z;\n\tmov.b32 {p, z}, %1;\n\tmov.b32 {q, z}, %2;\n\t"
        "fma.rn.f32.bf16 %0, p, q, %3;\n\t}"
        : "=f"(f)
        : "r"(a), "r"(c), "f"(addend));
    const float want_f = __fmaf_rn(widen(a), widen(c), addend);
    if (__float_as_uint(f) != __float_as_uint(want_f)) ++(f != f && want_f != want_f ? n[FMA] : b[FMA]);
  }
  for (int k = 0; k < NCHECK; ++k) {
    if (b[k]) atomicAdd(bad + k, b[k]);
    if (n[k]) atomicAdd(nan_only + k, n[k]);
  }
}

int main() {
  unsigned long long *bad = nullptr, *nan_only = nullptr;
  if (cudaMalloc(&bad, NCHECK * 8) != cudaSuccess || cudaMalloc(&nan_only, NCHECK * 8) != cudaSuccess) return 2;
  cudaMemset(bad, 0, NCHECK * 8);
  cudaMemset(nan_only, 0, NCHECK * 8);
  check_pairs<<<148 * 8, 256>>>(bad, nan_only);
  unsigned long long hb[NCHECK], hn[NCHECK];
  if (cudaMemcpy(hb, bad, sizeof hb, cudaMemcpyDeviceToHost) != cudaSuccess ||
      cudaMemcpy(hn, nan_only, sizeof hn, cudaMemcpyDeviceToHost) != cudaSuccess) {
    printf("cuda error: %s\n", cudaGetErrorString(cudaGetLastError()));
    return 2;
  }
  const char* names[NCHECK] = {"add.rn.bf16x2", "mul.rn.bf16x2", "fma.rn.f32.bf16(y,s,-0)", "fma.rn.f32.bf16(a,a,c)",
                               "fma.rn.f32.bf16(a,b,c)", "max.xorsign.abs.bf16x2"};
  unsigned long long total = 0;
  for (int k = 0; k < NCHECK; ++k) {
    printf("%s=%llu/%llu ", names[k], hb[k], hn[k]);
    total += hb[k];
  }
  printf("\n");
  return total == 0 ? 0 : 1;
}
