// Common device helpers for the sm_100a kernels of vllm_musa_b200.
//
// Everything here is plain CUDA C++ / inline PTX written for Blackwell (sm_100a):
// vector types for 128-bit global accesses, warp/block reductions, mbarrier and
// TMA (cp.async.bulk[.tensor]) wrappers, and the bounded-wait primitive every
// spin in this code base goes through.  A bounded wait never traps: when its
// budget runs out it records an error code in the error word the launcher passed
// in (one int per device, owned by vllm_musa_b200.ops._ext) and returns false, so
// the kernel can unwind, release TMEM and exit; the host reads the word after
// synchronising and raises.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define B200_DEVICE __device__ __forceinline__
#define B200_HOST_DEVICE __host__ __device__ __forceinline__

namespace b200 {

// ----------------------------------------------------------------------------------------------
// Error word codes:
//   1 = mbarrier wait timed out (TMA / MMA pipeline)
//   2 = peer flag wait timed out (communicator barrier)
//   3 = bad argument detected on device (index out of range) - access skipped
// ----------------------------------------------------------------------------------------------
enum ErrorCode : int {
  kErrNone = 0,
  kErrMbarTimeout = 1,
  kErrPeerTimeout = 2,
  kErrBadIndex = 3,
};

B200_DEVICE void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}
B200_DEVICE bool error_raised(const int* err) { return err && *((volatile const int*)err) != 0; }

// Wall budget of one bounded wait, in SM clock cycles (~1 s at 2 GHz).
constexpr long long kWaitBudgetCycles = 2000000000LL;

// ----------------------------------------------------------------------------------------------
// Vector helpers
// ----------------------------------------------------------------------------------------------
struct alignas(16) bf16x8 {
  __nv_bfloat162 v[4];
};

B200_DEVICE float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }
B200_DEVICE __nv_bfloat16 f2bf(float x) { return __float2bfloat16_rn(x); }

B200_DEVICE void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

B200_DEVICE uint4 pack8(const float (&f)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

// 2^x with the PTX ex2.approx.ftz instruction (the SFU's base-2 exponential; results below
// the normal range flush to zero, which softmax weights can afford).
B200_DEVICE float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

B200_DEVICE uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ----------------------------------------------------------------------------------------------
// Reductions (32-wide warps)
// ----------------------------------------------------------------------------------------------
B200_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

B200_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; `red` must hold >= 32 floats.  All threads get the result.
B200_DEVICE float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = (lane < nwarps) ? red[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

B200_DEVICE float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = (lane < nwarps) ? red[lane] : -INFINITY;
  t = warp_max(t);
  return t;
}

// ----------------------------------------------------------------------------------------------
// Shared-memory address / mbarrier
// ----------------------------------------------------------------------------------------------
B200_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

B200_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

B200_DEVICE void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

B200_DEVICE void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

B200_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

B200_DEVICE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

B200_DEVICE bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and records kErrMbarTimeout) when the
// budget runs out or another warp already raised an error.  The error word lives in global
// memory: it is polled only every 32nd failed try (a volatile load is an L2 round trip, and a
// pipeline hand-off waiting behind one notices its phase that much later).
B200_DEVICE bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t n = 1;; ++n) {
    if (mbar_try_wait(a, parity)) return true;
    if ((n & 31) == 0) {
      if (clock64() - t0 > kWaitBudgetCycles) {
        record_error(err, kErrMbarTimeout);
        return false;
      }
      if (error_raised(err)) return false;
    }
  }
}

// ----------------------------------------------------------------------------------------------
// TMA (bulk tensor copies).  No cluster multicast anywhere in this code base.
// ----------------------------------------------------------------------------------------------
B200_DEVICE void tma_prefetch_desc(const void* desc) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(desc)) : "memory");
}

B200_DEVICE void tma_load_2d(void* smem_dst, const void* desc, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// ---- thread-block clusters
B200_DEVICE uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
B200_DEVICE void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}
// shared::cluster address of `smem_addr` (a shared::cta address) in CTA `rank` of the cluster
B200_DEVICE uint32_t mapa_shared(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
B200_DEVICE void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
// TMA load issued by either CTA of a pair; completion bytes go to the mbarrier at the given
// shared::cluster address (the leader's).  Not a multicast load.
B200_DEVICE void tma_load_2d_pair(void* smem_dst, const void* desc, uint32_t bar_cluster_addr,
                                  int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(bar_cluster_addr), "r"(x), "r"(y)
      : "memory");
}

B200_DEVICE void tma_load_2d_hint(void* smem_dst, const void* desc, uint64_t* bar, int x, int y,
                                  uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

B200_DEVICE void tma_load_3d(void* smem_dst, const void* desc, uint64_t* bar, int x, int y,
                             int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Untiled bulk copy global->shared.  Both addresses 16-byte aligned, bytes % 16 == 0.
B200_DEVICE void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

B200_DEVICE uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

B200_DEVICE uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ----------------------------------------------------------------------------------------------
// cp.async (Ampere-style, 16B) for gathers that TMA cannot express cheaply.
// ----------------------------------------------------------------------------------------------
B200_DEVICE void cp_async16(void* smem, const void* gmem, bool pred = true) {
  const int sz = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(sz)
               : "memory");
}
B200_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
B200_DEVICE void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

B200_DEVICE int elect_one_lane() { return (threadIdx.x & 31) == 0; }

// Programmatic dependent launch: allow the next kernel of the stream (if it was launched with
// programmatic serialization, e.g. the GEMMs) to begin its prologue now.  It still waits for
// this grid to finish (griddepcontrol.wait) before reading what this grid writes.
B200_DEVICE void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

}  // namespace b200

#include "host_check.h"
