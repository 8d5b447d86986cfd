// The tensor-core ceiling of the MQA logits kernel: one CTA per SM, one lane issuing tcgen05.mma
// back to back from shared-memory operands in the kernel's own layout (128-byte swizzle, K-major)
// into two TMEM accumulators, with no copies and no epilogue.
//
//   kind::f8f6f4 M=128 N=256 K=32 (e4m3 x e4m3 -> f32): the MQA's instruction descriptor (MQ_IDESC),
//     key operand rotating over 6 stages and the query operand over 2, one commit a tile of 4 MMAs;
//   kind::f16    M=128 N=256 K=16 (bf16 x bf16 -> f32): the same loop in bf16, for comparison with
//     the cuBLAS bf16 GEMM rate.
//
// Prints one line per kind: name TFLOP/s (best of 3) and the SM clock over the launch (clock64 over
// globaltimer); exit status 0 when every bounded wait ended. Built and run by
// tests/test_gpu_tcgen05_rate.py.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

#include "glmkv_mqa.cuh"

using namespace glmkv;

constexpr int A_ST = 6, B_ST = 2, N = 256;
constexpr int OPBYTES = (A_ST * 128 + B_ST * N) * 128;

template <int KIND>  // 0: f8f6f4 (e4m3), 1: f16 (bf16)
__global__ void __launch_bounds__(128, 1) mma_loop(int iters, unsigned long long* clk, int* err) {
  extern __shared__ __align__(1024) u8 smem_raw[];
  __shared__ __align__(8) unsigned long long done, tile_bar[2];
  __shared__ uint32_t tbase;
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  u8* sg = smem_raw + (sbase - smem_u32(smem_raw));
  const int tid = threadIdx.x;
  // operand bytes without NaN or infinity codes: e4m3 exponent field <= 6; bf16 values +-(1 .. 2) 2^-7
  for (int i = tid; i < OPBYTES; i += blockDim.x) {
    const uint32_t h = (uint32_t)i * 2654435761u;
    sg[i] = KIND == 0 ? (u8)((h >> 24) & 0xB7) : (u8)((i & 1) ? (0x3C | (((h >> 28) & 1) << 7)) : (h >> 24));
  }
  if (tid == 0) {
    mbar_init(smem_u32(&done), 1);
    mbar_init(smem_u32(&tile_bar[0]), 1);
    mbar_init(smem_u32(&tile_bar[1]), 1);
    mbar_init_fence();
  }
  if (tid < 32) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tbase)), "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the operands, for the tensor cores
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tbase;
  if (tid == 0) {
    const uint32_t idesc = KIND == 0 ? MQ_IDESC
                                     : ((1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
                                        ((uint32_t)(128 >> 4) << 24));
    const uint64_t c0 = clock64(), t0 = global_ns();
    for (int it = 0; it < iters; ++it) {
      if (it >= 2) {  // the tile two back has completed (the kernel's two accumulators)
        if (!mbar_wait_bounded(smem_u32(&tile_bar[it & 1]), ((it >> 1) - 1) & 1, WAIT_LIMIT_NS)) {
          atomicOr(err, 1);
          break;
        }
        tc_fence_after();
      }
      const uint64_t adesc = sw128_desc(sbase + (it % A_ST) * 128 * 128);
      const uint64_t bdesc = sw128_desc(sbase + A_ST * 128 * 128 + ((it / 16) % B_ST) * N * 128);
      const uint32_t d = tmem + (it & 1) * N;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        if (KIND == 0)
          tc_mma(d, adesc + 2 * kk, bdesc + 2 * kk, idesc, kk > 0);
        else
          asm volatile(
              "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
              "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
              "l"(adesc + 2 * kk), "l"(bdesc + 2 * kk), "r"(idesc), "r"(kk)
              : "memory");
      }
      tc_commit(smem_u32(&tile_bar[it & 1]));
    }
    tc_commit(smem_u32(&done));
    if (!mbar_wait_bounded(smem_u32(&done), 0, WAIT_LIMIT_NS)) atomicOr(err, 2);
    if (blockIdx.x == 0) {
      clk[0] = clock64() - c0;
      clk[1] = global_ns() - t0;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid < 32) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
}

template <int KIND>
int run(const char* name, int sms, int iters, unsigned long long* clk, int* err) {
  const int smem = 1024 + OPBYTES;
  if (cudaFuncSetAttribute(mma_loop<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return 1;
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  double best = 0, mhz = 0;
  for (int rep = 0; rep < 3; ++rep) {
    cudaEventRecord(e0);
    mma_loop<KIND><<<sms, 128, smem>>>(iters, clk, err);
    cudaEventRecord(e1);
    if (cudaEventSynchronize(e1) != cudaSuccess) {
      printf("%s: %s\n", name, cudaGetErrorString(cudaGetLastError()));
      return 1;
    }
    float ms;
    cudaEventElapsedTime(&ms, e0, e1);
    unsigned long long h[2];
    cudaMemcpy(h, clk, sizeof h, cudaMemcpyDeviceToHost);
    const double flop = 2.0 * 128 * N * (KIND == 0 ? 128 : 64) * (double)iters * sms;  // K of 4 MMAs
    if (flop / ms / 1e9 > best) best = flop / ms / 1e9, mhz = (double)h[0] / (double)h[1] * 1e3;
  }
  printf("%s %.1f TFLOP/s %.0f MHz\n", name, best, mhz);
  return 0;
}

int main() {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  unsigned long long* clk = nullptr;
  int* err = nullptr;
  if (cudaMalloc(&clk, 16) != cudaSuccess || cudaMalloc(&err, 4) != cudaSuccess) return 2;
  cudaMemset(err, 0, 4);
  int bad = run<0>("f8f6f4_e4m3_m128n256", sms, 40000, clk, err);
  bad |= run<1>("f16_bf16_m128n256", sms, 20000, clk, err);
  int herr = 0;
  cudaMemcpy(&herr, err, 4, cudaMemcpyDeviceToHost);
  printf("wait_errors %d\n", herr);
  return bad || herr ? 1 : 0;
}
