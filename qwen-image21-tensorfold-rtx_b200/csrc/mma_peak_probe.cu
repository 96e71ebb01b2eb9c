// Roofline probe: the tcgen05 issue-rate ceiling of one CTA per SM (no loads, zero operands).
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -o mma_peak_probe mma_peak_probe.cu   (build.py --probe)
//
// Each CTA allocates TMEM, then one thread issues `iters` back-to-back tcgen05.mma (M=128, N=256) of a kind and
// waits for them through a tcgen05.commit. The reported TFLOP/s is the dense-MMA ceiling the GEMM kernels are
// measured against (it includes no operand traffic, so a real GEMM cannot exceed it). The final wait is bounded.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

namespace {

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint64_t desc_sw128(const void* p) {
  const uint64_t a = su32(p);
  return ((a & 0x3FFFFull) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

template <int KIND>  // 0: kind::mxf4nvf4 block16 (K=64), 1: kind::f8f6f4 e4m3 (K=32)
__global__ void __launch_bounds__(128, 1) probe(int iters, unsigned long long* cycles, int* err) {
  extern __shared__ uint8_t raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)raw + 1023) & ~(uintptr_t)1023);
  __shared__ uint64_t bar;
  __shared__ uint32_t slot;
  for (int i = threadIdx.x; i < 48 * 1024 / 16; i += blockDim.x) ((uint4*)sm)[i] = make_uint4(0, 0, 0, 0);
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&bar)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (threadIdx.x < 32) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(su32(&slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tm = slot;
  if (threadIdx.x == 0) {
    const uint32_t idesc = KIND == 0 ? ((1u << 7) | (1u << 10) | (32u << 17) | (8u << 24))
                                     : ((1u << 4) | (32u << 17) | (8u << 24));
    const unsigned long long t0 = clock64();
    for (int i = 0; i < iters; ++i) {
      const int kb = i & 3;
      if (KIND == 0)
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
            ::"r"(tm), "l"(desc_sw128(sm + kb * 32)), "l"(desc_sw128(sm + 16384 + kb * 32)), "r"(idesc),
            "r"((uint32_t)(i > 0)), "r"(tm + 256), "r"(tm + 272));
      else
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}"
            ::"r"(tm), "l"(desc_sw128(sm + kb * 32)), "l"(desc_sw128(sm + 16384 + kb * 32)), "r"(idesc),
            "r"((uint32_t)(i > 0)));
    }
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(&bar))
                 : "memory");
    unsigned long long g0, g1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g0));
    uint32_t ok = 0;
    while (!ok) {
      asm volatile(
          "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\tselp.u32 %0, 1, 0, p;\n\t}"
          : "=r"(ok)
          : "r"(su32(&bar))
          : "memory");
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g1));
      if (!ok && g1 - g0 > 1000000000ull) {
        atomicExch(err, 1);
        break;
      }
    }
    cycles[blockIdx.x] = clock64() - t0;
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (threadIdx.x < 32) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tm));
  }
}

template <int KIND>
int run(const char* name, int sms, unsigned long long* dcyc, int* derr) {
  const int iters = 8192, smem = 49 * 1024;
  cudaFuncSetAttribute(probe<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  probe<KIND><<<sms, 128, smem>>>(iters, dcyc, derr);  // warm-up
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  cudaEventRecord(a);
  probe<KIND><<<sms, 128, smem>>>(iters, dcyc, derr);
  cudaEventRecord(b);
  if (cudaEventSynchronize(b) != cudaSuccess) return 1;
  float ms = 0;
  cudaEventElapsedTime(&ms, a, b);
  unsigned long long h[1024];
  cudaMemcpy(h, dcyc, sms * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
  double avg = 0;
  for (int i = 0; i < sms; ++i) avg += (double)h[i];
  avg /= sms;
  int e = 0;
  cudaMemcpy(&e, derr, sizeof(int), cudaMemcpyDeviceToHost);
  const double flop = 2.0 * 128 * 256 * (KIND == 0 ? 64 : 32) * iters * sms;
  printf("%-34s %7.1f cycles/MMA  %8.0f TFLOP/s  (%d SMs, kernel %.3f ms, wait-timeout=%d)\n", name, avg / iters,
         flop / (ms * 1e-3) / 1e12, sms, ms, e);
  return e;
}

}  // namespace

int main() {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  unsigned long long* dcyc;
  int* derr;
  cudaMalloc(&dcyc, 1024 * sizeof(unsigned long long));
  cudaMalloc(&derr, sizeof(int));
  cudaMemset(derr, 0, sizeof(int));
  int bad = run<0>("mxf4nvf4 block16 M128 N256 K64", sms, dcyc, derr);
  bad |= run<1>("f8f6f4 e4m3 M128 N256 K32", sms, dcyc, derr);
  return bad;
}
