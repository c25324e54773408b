// Dense int8 tensor-core peak of this GPU (the roofline denominator of the GEMM).
//
// One CTA per SM issues back-to-back tcgen05.mma.cta_group::1.kind::i8 (M=128,
// N=256, K=32) from operands resident in shared memory into one TMEM
// accumulator; no loads, no epilogue. Reported: int8 TOPS (2 ops per MAC) over
// the whole GPU, timed with CUDA events around the launch.
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -o i8_peak i8_peak.cu
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

constexpr int N = 256, M = 128;
constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint64_t desc(uint32_t a) {
  return (uint64_t)((a >> 4) & 0x3fff) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

__global__ void __launch_bounds__(128, 1) peak_kernel(int iters, unsigned* out) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar;
  __shared__ uint32_t tslot;
  for (int i = threadIdx.x; i < (M + N) * 128 / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(smem)[i] = i * 2654435761u;
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bar)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (threadIdx.x < 32) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tslot)), "r"(256));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tslot;
  if (threadIdx.x == 0) {
    const uint32_t a = smem_u32(smem), b = smem_u32(smem + M * 128);
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int k = 0; k < 4; ++k)
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(
                tmem),
            "l"(desc(a + 32 * k)), "l"(desc(b + 32 * k)), "r"(IDESC), "r"((it | k) ? 1u : 0u));
    }
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(&bar))
                 : "memory");
    uint32_t ok = 0;
    const long long t0 = clock64();
    while (!ok && clock64() - t0 < 8000000000ll)
      asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                   : "=r"(ok)
                   : "r"(smem_u32(&bar)));
    if (!ok) atomicAdd(out, 1u);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (threadIdx.x < 32) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256));
  }
}

int main() {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  unsigned* timeouts = nullptr;
  cudaMalloc(&timeouts, sizeof(unsigned));
  cudaMemset(timeouts, 0, sizeof(unsigned));
  const int smem = (M + N) * 128 + 1024;
  cudaFuncSetAttribute(peak_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  const int iters = 20000;
  peak_kernel<<<sms, 128, smem>>>(1000, timeouts);
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  float best = 1e30f;
  for (int r = 0; r < 5; ++r) {
    cudaEventRecord(a);
    peak_kernel<<<sms, 128, smem>>>(iters, timeouts);
    cudaEventRecord(b);
    cudaEventSynchronize(b);
    float ms = 0;
    cudaEventElapsedTime(&ms, a, b);
    if (ms < best) best = ms;
  }
  unsigned h = 0;
  cudaMemcpy(&h, timeouts, sizeof h, cudaMemcpyDeviceToHost);
  const cudaError_t e = cudaDeviceSynchronize();
  const double ops = 2.0 * M * N * 32 * 4.0 * iters * sms;
  printf("{\"i8_dense_tops\": %.1f, \"ms\": %.3f, \"sms\": %d, \"mma\": \"tcgen05 kind::i8 M=%d N=%d K=32, operands in smem\", "
         "\"timeouts\": %u, \"status\": \"%s\"}\n",
         ops / (best * 1e-3) / 1e12, best, sms, M, N, h, cudaGetErrorString(e));
  return (e != cudaSuccess || h) ? 1 : 0;
}
