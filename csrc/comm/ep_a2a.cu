// Expert-parallel all-to-all over NVSwitch peer memory (dispatch -> grouped experts -> combine),
// for MoE layers whose attention is tensor-parallel.
//
// After attention every rank holds all T tokens' (normalised) hidden states.  Rank r owns the
// token shard [r*P, r*P+P) (P = ceil(T / N), the two-shot row chunk):
//
//   ep_dispatch_kernel   one warp per shard token: the ranks owning its top-k experts are
//                        found with warp ballots; the token row is stored ONCE per destination
//                        rank (16-byte stores into that rank's receive region for this source,
//                        slot from a local atomic counter) together with the (local expert id,
//                        weight) pairs that rank serves (-1 elsewhere) and the token's shard
//                        index.  Rows travel over NVLink by plain stores; no TMA, no multicast.
//   ep_exchange_kernel   one CTA: publishes the per-destination row counts into each peer's
//                        count slots, then an epoch barrier (release / acquire at system scope,
//                        bounded by a clock budget -> error word) so every rank's receive region
//                        is complete; resets the local send counters.
//   ep_mask_kernel       marks receive rows beyond each source's count as empty (-1 experts).
//   (experts)            the grouped MoE GEMMs run on the receive region as [N * cap, k]
//                        routing (moe_align / moe_gather / grouped GEMM with SwiGLU).
//   ep_return_kernel     per received row: the weighted sum of its local experts' outputs is
//                        stored straight into block `me` of the SOURCE rank's all-reduce staging
//                        slot, at the token's shard row.
// The source rank then runs the two-shot all-reduce kernel in local-source mode over those N
// blocks (+ residual, RMSNorm, all-gather of the normalised rows): the combine and the
// reduction share one pass.  Buffers are single-buffered: consecutive layers are separated by
// the all-reduce's barriers.
//
// Reference counterpart: DeepEP dispatch/combine used through vLLM's all2all manager
// (reference patches 0052 / 0112, vllm_musa/model_executor/layers/fused_moe/
// unquantized_fused_moe_method.py:39-75); the reference has no kernel source for it.
#include <algorithm>

#include "../b200_kernels.h"
#include "../common/common.cuh"
#include "custom_ar.h"

namespace b200 {
namespace ep {

B200_DEVICE void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
B200_DEVICE uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void ep_dispatch_kernel(A2AParams p) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= p.Tc) return;
  const int t = warp;  // shard-local token
  const int k = p.k;
  int e = -1, d = -1;
  float w = 0.f;
  if (lane < k) {
    e = p.ids[(size_t)t * k + lane];
    w = p.w[(size_t)t * k + lane];
    d = (e >= 0 && e < p.E_local * p.world) ? e / p.E_local : -1;
  }
  const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(p.x) + (size_t)(p.row0 + t) * p.ldx;
  const int nvec = p.H / 8;
  for (int dst = 0; dst < p.world; ++dst) {
    const unsigned mask = __ballot_sync(0xffffffffu, d == dst);
    if (!mask) continue;
    int slot = 0;
    if (lane == 0) slot = atomicAdd(&p.send_cnt[dst], 1);
    slot = __shfl_sync(0xffffffffu, slot, 0);
    if (slot >= p.cap) {  // cannot happen with cap >= shard rows; never write out of bounds
      if (lane == 0) record_error(p.err, kErrBadIndex);
      continue;
    }
    const size_t row = (size_t)p.rank * p.cap + slot;  // this source's region at `dst`
    uint4* xd = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.recv_x[dst]) + row * p.H);
    const uint4* xs = reinterpret_cast<const uint4*>(src);
    for (int c = lane; c < nvec; c += 32) xd[c] = xs[c];
    if (lane < k) {
      p.recv_ids[dst][row * k + lane] = d == dst ? e - dst * p.E_local : -1;
      p.recv_w[dst][row * k + lane] = w;
    }
    if (lane == 0) p.recv_tok[dst][row] = t;
  }
  __threadfence_system();  // peer stores visible before the exchange barrier publishes them
}

__global__ void ep_exchange_kernel(A2AParams p) {
  __shared__ uint32_t epoch_s;
  if (threadIdx.x == 0) epoch_s = ++(*p.epoch);
  __syncthreads();
  const uint32_t epoch = epoch_s;
  const int q = threadIdx.x;
  if (q < p.world) {
    // my row count for q goes into q's count slot for source `rank`
    p.recv_cnt[q][p.rank] = p.send_cnt[q];
    p.send_cnt[q] = 0;
    __threadfence_system();
    st_release_sys(p.flags[q] + p.rank, epoch);
    const uint32_t* mine = p.flags[p.rank] + q;
    const long long t0 = clock64();
    for (uint32_t spin = 1; (int32_t)(ld_acquire_sys(mine) - epoch) < 0; ++spin) {
      if ((spin & 31) != 0) continue;  // error word / clock every 32nd poll
      if (clock64() - t0 > kWaitBudgetCycles) {
        record_error(p.err, kErrPeerTimeout);
        break;
      }
      if (error_raised(p.err)) break;
    }
  }
}

__global__ void ep_mask_kernel(A2AParams p) {
  const int src = blockIdx.y;
  const int n = p.recv_cnt[p.rank][src];
  int32_t* ids = p.recv_ids[p.rank] + (size_t)src * p.cap * p.k;
  for (int i = n * p.k + blockIdx.x * blockDim.x + threadIdx.x; i < p.cap * p.k;
       i += gridDim.x * blockDim.x)
    ids[i] = -1;
}

// y: [max_rows, H] expert outputs; pos: [N * cap, k] rows of y for each (received row, slot)
__global__ void ep_return_kernel(A2AParams p, const __nv_bfloat16* __restrict__ y,
                                 const int32_t* __restrict__ pos) {
  const int r = blockIdx.x;  // received row
  const int src = r / p.cap, slot = r - src * p.cap;
  if (slot >= p.recv_cnt[p.rank][src]) return;
  const int k = p.k;
  const float* w = p.recv_w[p.rank] + (size_t)r * k;
  const int32_t* ps = pos + (size_t)r * k;
  const int t = p.recv_tok[p.rank][r];
  __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.staging[src]) +
                       ((size_t)p.rank * p.rs_rows + t) * p.H;
  for (int c = threadIdx.x; c < p.H / 8; c += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < k; ++j) {
      const int yr = ps[j];
      if (yr < 0) continue;
      float f[8];
      unpack8(reinterpret_cast<const uint4*>(y + (size_t)yr * p.H)[c], f);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += w[j] * f[q];
    }
    reinterpret_cast<uint4*>(dst)[c] = pack8(acc);
  }
  __threadfence_system();
}

// ------------------------------------------------------------------------------ launchers
static void check(const A2AParams& p) {
  B200_REQUIRE(p.world >= 1 && p.world <= comm::kMaxRanks, "ep a2a: world size");
  B200_REQUIRE(p.k >= 1 && p.k <= 32, "ep a2a: top-k must be 1..32");
  B200_REQUIRE(p.H % 8 == 0, "ep a2a: hidden % 8");
  B200_REQUIRE(p.Tc <= p.cap, "ep a2a: shard larger than the receive capacity");
}

void run_dispatch(const A2AParams& p, cudaStream_t s) {
  check(p);
  if (p.Tc > 0) {
    ep_dispatch_kernel<<<(p.Tc + 3) / 4, 128, 0, s>>>(p);
    B200_CUDA_OK(cudaGetLastError());
    count_launch();
  }
  ep_exchange_kernel<<<1, 32, 0, s>>>(p);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
  ep_mask_kernel<<<dim3(std::max(1, std::min(64, p.cap * p.k / 256)), p.world), 256, 0, s>>>(p);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

void run_return(const A2AParams& p, const void* y, const int32_t* pos, cudaStream_t s) {
  check(p);
  ep_return_kernel<<<p.world * p.cap, 128, 0, s>>>(p, reinterpret_cast<const __nv_bfloat16*>(y), pos);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

}  // namespace ep
}  // namespace b200
