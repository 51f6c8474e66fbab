// Tiled TMA (cp.async.bulk.tensor.2d, 128-byte swizzle) -> shared-memory throughput probe.
//
// Each CTA runs `nprod` producer threads (lane 0 of warps 0..nprod-1), each with its own ring
// of `stages` mbarrier stages holding `per_stage` boxes of box_rows x 128 bytes.  mode 0: all
// CTAs walk one 32 MiB window (L2-resident); mode 1: each producer streams its own slice of a
// multi-GB buffer (HBM).  No cluster multicast.  Every wait is bounded and records an error.
// Built and driven by tma_probe.py.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include "common/tma_host.h"

__device__ __forceinline__ uint32_t sa(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__global__ void tbw_kernel(const __grid_constant__ CUtensorMap tm, int rows_total, int box_rows,
                           int per_stage, int stages, int iters, int mode, int* err, int nprod) {
  extern __shared__ __align__(1024) char smem_raw[];
  __shared__ __align__(8) uint64_t bars[4][16];
  const int copy_bytes = box_rows * 128;
  const int stage_bytes = copy_bytes * per_stage;
  if (threadIdx.x == 0) {
    for (int w = 0; w < nprod; ++w)
      for (int s = 0; s < stages; ++s)
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sa(&bars[w][s])));
    asm volatile("fence.mbarrier_init.release.cluster;");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tm) : "memory");
  }
  __syncthreads();
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) != 0 || w >= nprod) return;
  uint64_t* bar = bars[w];
  smem_raw[0] = smem_raw[0];
  char* mine = (char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023) + (size_t)w * stages * stage_bytes;
  uint32_t phase = 0;
  const int span = iters * per_stage * box_rows;
  int row = mode == 1 ? (blockIdx.x * nprod + w) * span : ((blockIdx.x * nprod + w) * 977 * box_rows) % rows_total;
  for (int i = 0; i < iters + stages; ++i) {
    const int s = i % stages;
    if (i >= stages) {
      uint32_t done = 0;
      long long n = 0;
      while (!done) {
        asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                     : "=r"(done) : "r"(sa(&bar[s])), "r"(phase) : "memory");
        if (++n > 20000000) { atomicExch(err, 1); return; }
      }
      if (s == stages - 1) phase ^= 1;
    }
    if (i < iters) {
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(&bar[s])), "r"(stage_bytes) : "memory");
      for (int p = 0; p < per_stage; ++p) {
        asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
                     ::"r"(sa(mine + (size_t)s * stage_bytes + p * copy_bytes)), "l"(&tm), "r"(sa(&bar[s])),
                       "r"(0), "r"(row) : "memory");
        row += box_rows;
        if (mode == 0 && row + box_rows > rows_total) row = 0;
      }
    }
  }
}

extern "C" int run_tbw(void* src, long long bytes, int grid, int box_rows, int per_stage,
                       int stages, int iters, int mode, float* ms, int* err_dev, int nprod) {
  const int rows_total = (int)(bytes / 128);
  CUtensorMap tm = b200::make_tma_2d(src, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 64, rows_total, 64,
                                     64, box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
  const int smem = box_rows * 128 * per_stage * stages * nprod + 1024;
  cudaFuncSetAttribute(tbw_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  tbw_kernel<<<grid, 32 * nprod, smem>>>(tm, rows_total, box_rows, per_stage, stages, iters, mode, err_dev, nprod);
  cudaEventRecord(a);
  tbw_kernel<<<grid, 32 * nprod, smem>>>(tm, rows_total, box_rows, per_stage, stages, iters, mode, err_dev, nprod);
  cudaEventRecord(b);
  cudaEventSynchronize(b);
  cudaEventElapsedTime(ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  return (int)cudaGetLastError();
}
