// NVSwitch peer-memory all-reduce fused with residual-add + RMSNorm, for tensor parallelism.
//
// Every rank owns an IPC-exported buffer holding (a) two staging slots that the preceding
// row-parallel GEMM writes its partial sums into, (b) two output slots, (c) barrier flags.
// Peers map each other's buffers (cudaIpcOpenMemHandle) and the kernels below read / write
// them with plain 16-byte loads and stores over NVLink: no NCCL call, no staging copy, and
// never a TMA (let alone multicast TMA) load from peer memory.
//
//  one-shot (small T):   start barrier; every rank reduces ALL rows from all peers' staging,
//                        adds the (replicated) residual, normalises, writes its local output.
//  two-shot (larger T):  start barrier; rank r reduces only its row chunk from all peers,
//                        adds the residual rows it owns (the residual stream stays
//                        row-sharded: rank r is the only writer of its rows), normalises, and
//                        stores the normalised rows into EVERY rank's output slot (the
//                        all-gather rides on posted P2P stores); end barrier.
// Barriers are per block: block b of every rank bumps its own epoch counter, publishes it to
// each peer's flag slot [phase][b][rank] with a release store, and spins (acquire loads,
// bounded by a clock budget) until all peers' slots for block b reach the epoch.  Slots
// alternate by call parity, so one start barrier also proves every peer finished the
// previous call (which is what frees the other parity's buffers).  On a timeout the kernel
// records kErrPeerTimeout in the error word and returns without touching the data.
//
// Reference counterpart: vllm_musa/jit_kernel/csrc/distributed/custom_all_reduce.mu:151-1126
// (flag barrier, 1-stage / 2-stage / 2-shot reduce, fused AR + RMSNorm variants) driven by
// vllm_musa/distributed/device_communicators/musa_jit_custom_all_reduce.py:440-1760.
#include <algorithm>

#include "../b200_kernels.h"
#include "../common/common.cuh"
#include <cuda_runtime.h>
#include <string.h>

#include "custom_ar.h"

namespace b200 {
namespace comm {

B200_DEVICE void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
B200_DEVICE uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Block-level barrier among the `world` ranks for block `b`.  Thread p (< world) signals
// rank p and waits for rank p's signal.  Returns false on timeout.
B200_DEVICE bool block_barrier(const ArParams& a, int phase, uint32_t epoch) {
  __shared__ int ok_all;
  if (threadIdx.x == 0) ok_all = 1;
  __syncthreads();
  const int b = blockIdx.x;
  if (threadIdx.x < a.world) {
    const int p = threadIdx.x;
    uint32_t* peer_slot = a.flags[p] + ((size_t)phase * kMaxBlocks + b) * kMaxRanks + a.rank;
    __threadfence_system();
    st_release_sys(peer_slot, epoch);
    const uint32_t* my_slot = a.flags[a.rank] + ((size_t)phase * kMaxBlocks + b) * kMaxRanks + p;
    const long long t0 = clock64();
    for (uint32_t spin = 1; (int32_t)(ld_acquire_sys(my_slot) - epoch) < 0; ++spin) {
      if ((spin & 31) != 0) continue;  // error word / clock every 32nd poll
      if (clock64() - t0 > kWaitBudgetCycles) {
        record_error(a.err, kErrPeerTimeout);
        ok_all = 0;
        break;
      }
      if (error_raised(a.err)) {
        ok_all = 0;
        break;
      }
    }
  }
  __syncthreads();
  return ok_all != 0;
}

// One row: sum the row over all ranks' staging, add residual, normalise.  VPT vectors of 8
// bf16 per thread.  Writes residual (if any) and returns normalised values in `o`.
template <int VPT, bool kNorm>
B200_DEVICE void reduce_row(const ArParams& a, int row, int r0, float (&o)[VPT][8], float* red) {
  const int nvec = a.H / 8;
  float v[VPT][8];
#pragma unroll
  for (int i = 0; i < VPT; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
  // peers' staging (row-major [T, H]) or, after an epilogue reduce-scatter, block p of the
  // local staging slot.  All ranks' vectors are loaded before any is summed, so the NVLink
  // round trips overlap instead of running one peer after another.
  const uint4* src[kMaxRanks];
#pragma unroll
  for (int p = 0; p < kMaxRanks; ++p) {
    const int pp = p < a.world ? p : 0;
    src[p] = reinterpret_cast<const uint4*>(
        a.rs_rows > 0 ? reinterpret_cast<const __nv_bfloat16*>(a.staging[a.rank]) +
                            ((size_t)pp * a.rs_rows + (row - r0)) * a.H
                      : reinterpret_cast<const __nv_bfloat16*>(a.staging[pp]) + (size_t)row * a.H);
  }
  // (rows of up to 2 vectors per thread keep every rank's loads in registers at once; wider
  // rows take one vector index at a time to stay within the register budget)
#pragma unroll(VPT <= 2 ? VPT : 1)
  for (int i = 0; i < VPT; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nvec) {
      uint4 t[kMaxRanks];
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p)
        if (p < a.world) t[p] = src[p][c];
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p) {
        if (p < a.world) {
          float f[8];
          unpack8(t[p], f);
#pragma unroll
          for (int j = 0; j < 8; ++j) v[i][j] += f[j];
        }
      }
    }
  }
  float ss = 0.f;
  if (a.residual) {
    uint4* rr = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.residual) +
                                         (size_t)row * a.H);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < nvec) {
        float r[8];
        unpack8(rr[c], r);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] += r[j];
        const uint4 pk = pack8(v[i]);
        rr[c] = pk;
        unpack8(pk, v[i]);
      }
    }
  }
  if constexpr (kNorm) {
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < nvec)
#pragma unroll
        for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
    ss = block_sum(ss, red);
    const float inv = rsqrtf(ss / a.H + a.eps);
    const uint4* wr = reinterpret_cast<const uint4*>(a.weight);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < nvec) {
        float w[8];
        unpack8(wr[c], w);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[i][j] = v[i][j] * inv * w[j];
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) o[i][j] = v[i][j];
  }
}

template <int VPT, bool kNorm, bool kTwoShot>
__global__ void __launch_bounds__(512) fused_ar_kernel(ArParams a) {
  __shared__ float red[32];
  __shared__ uint32_t epoch_s;
  if (threadIdx.x == 0) {
    epoch_s = a.epochs[blockIdx.x] + 1;
    a.epochs[blockIdx.x] = epoch_s;
  }
  __syncthreads();
  const uint32_t epoch = epoch_s;
  if (!block_barrier(a, a.parity, epoch)) return;
  const int nvec = a.H / 8;
  int r0 = 0, r1 = a.T;
  if (kTwoShot) {
    const int per = (a.T + a.world - 1) / a.world;
    r0 = min(a.T, a.rank * per);
    r1 = min(a.T, r0 + per);
  }
  for (int row = r0 + blockIdx.x; row < r1; row += gridDim.x) {
    float o[VPT][8];
    reduce_row<VPT, kNorm>(a, row, r0, o, red);
    const int nout = kTwoShot ? a.world : 1;
    for (int q = 0; q < nout; ++q) {
      const int dst_rank = kTwoShot ? (a.rank + q) % a.world : a.rank;
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.out[dst_rank]) +
                                            (size_t)row * a.H);
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int c = threadIdx.x + i * blockDim.x;
        if (c < nvec) dst[c] = pack8(o[i]);
      }
    }
  }
  if (kTwoShot || a.end_barrier) block_barrier(a, 2 + a.parity, epoch);
}

// Variant for many rows per rank (large T, two-shot or one-shot): one WARP per row and eight rows per
// block, so every block keeps eight rows' peer loads in flight instead of walking one row at a
// time with block-wide reductions.  Lane l owns the 8-element vectors l, l+32, ... of the row
// (VPW of them); peer loads are issued CH vectors x NPEER ranks at a time (16 16-byte loads
// per lane per round trip), accumulated in fp32, the residual added and rounded to bf16 (as
// the unfused add would), the row normalised with a warp reduction and stored into every
// rank's output slot.  Same barriers, flags and buffers as fused_ar_kernel.
constexpr int kWarpRowThreads = 256;

template <int VPW, int NPEER, bool kNorm, bool kTwoShot>
__global__ void __launch_bounds__(kWarpRowThreads) fused_ar_warp_kernel(ArParams a) {
  constexpr int CH = 16 / NPEER;  // vectors per round trip (x NPEER loads in flight)
  static_assert(VPW % CH == 0, "vectors per lane must be a multiple of the chunk");
  __shared__ uint32_t epoch_s;
  if (threadIdx.x == 0) {
    epoch_s = a.epochs[blockIdx.x] + 1;
    a.epochs[blockIdx.x] = epoch_s;
  }
  __syncthreads();
  const uint32_t epoch = epoch_s;
  if (!block_barrier(a, a.parity, epoch)) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kWarps = kWarpRowThreads / 32;
  const int nvec = a.H / 8;
  // two-shot: this rank's row chunk, stored to every rank; one-shot: every row, stored locally
  const int per = kTwoShot ? (a.T + NPEER - 1) / NPEER : a.T;
  const int r0 = kTwoShot ? min(a.T, a.rank * per) : 0, r1 = min(a.T, r0 + per);
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  for (int row = r0 + blockIdx.x * kWarps + warp; row < r1; row += gridDim.x * kWarps) {
    uint4 packed[VPW];
#pragma unroll
    for (int i0 = 0; i0 < VPW; i0 += CH) {
      uint4 t[NPEER][CH];
#pragma unroll
      for (int p = 0; p < NPEER; ++p) {
        const __nv_bfloat16* base =
            a.rs_rows > 0 ? reinterpret_cast<const __nv_bfloat16*>(a.staging[a.rank]) +
                                ((size_t)p * a.rs_rows + (row - r0)) * a.H
                          : reinterpret_cast<const __nv_bfloat16*>(a.staging[p]) +
                                (size_t)row * a.H;
        const uint4* src = reinterpret_cast<const uint4*>(base);
#pragma unroll
        for (int k = 0; k < CH; ++k) {
          const int c = lane + 32 * (i0 + k);
          t[p][k] = c < nvec ? src[c] : zero;
        }
      }
#pragma unroll
      for (int k = 0; k < CH; ++k) {
        const int c = lane + 32 * (i0 + k);
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int p = 0; p < NPEER; ++p) {
          float f[8];
          unpack8(t[p][k], f);
#pragma unroll
          for (int j = 0; j < 8; ++j) v[j] += f[j];
        }
        if (a.residual && c < nvec) {
          uint4* rr = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.residual) +
                                               (size_t)row * a.H);
          float r[8];
          unpack8(rr[c], r);
#pragma unroll
          for (int j = 0; j < 8; ++j) v[j] += r[j];
          packed[i0 + k] = pack8(v);
          rr[c] = packed[i0 + k];
        } else {
          packed[i0 + k] = pack8(v);
        }
      }
    }
    float inv = 1.f;
    if constexpr (kNorm) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < VPW; ++i) {
        if (lane + 32 * i < nvec) {
          float f[8];
          unpack8(packed[i], f);
#pragma unroll
          for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
        }
      }
      ss = warp_sum(ss);
      inv = rsqrtf(ss / a.H + a.eps);
    }
#pragma unroll
    for (int i = 0; i < VPW; ++i) {
      const int c = lane + 32 * i;
      if (c >= nvec) continue;
      uint4 ov = packed[i];
      if constexpr (kNorm) {
        float f[8], w[8];
        unpack8(packed[i], f);
        unpack8(reinterpret_cast<const uint4*>(a.weight)[c], w);
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = f[j] * inv * w[j];
        ov = pack8(f);
      }
#pragma unroll
      for (int q = 0; q < (kTwoShot ? NPEER : 1); ++q) {
        const int dst_rank = (a.rank + q) % NPEER;
        reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.out[dst_rank]) +
                                 (size_t)row * a.H)[c] = ov;
      }
    }
  }
  if (kTwoShot || a.end_barrier) block_barrier(a, 2 + a.parity, epoch);
}

template <int VPW, bool kNorm, bool kTwoShot>
static void launch_warp_rows(const ArParams& a, cudaStream_t s) {
  if (a.world == 2)
    fused_ar_warp_kernel<VPW, 2, kNorm, kTwoShot><<<a.blocks, kWarpRowThreads, 0, s>>>(a);
  else if (a.world == 4)
    fused_ar_warp_kernel<VPW, 4, kNorm, kTwoShot><<<a.blocks, kWarpRowThreads, 0, s>>>(a);
  else
    fused_ar_warp_kernel<VPW, 8, kNorm, kTwoShot><<<a.blocks, kWarpRowThreads, 0, s>>>(a);
}

template <bool kNorm, bool kTwoShot>
static void dispatch_warp_rows(const ArParams& a, int nvec, cudaStream_t s) {
  if (nvec <= 32 * 8)
    launch_warp_rows<8, kNorm, kTwoShot>(a, s);
  else
    launch_warp_rows<16, kNorm, kTwoShot>(a, s);
}

template <bool kNorm, bool kTwoShot>
static void launch(const ArParams& a, int threads, int vpt, int blocks, cudaStream_t s) {
#define B200_AR(V) fused_ar_kernel<V, kNorm, kTwoShot><<<blocks, threads, 0, s>>>(a)
  if (vpt <= 1)
    B200_AR(1);
  else if (vpt <= 2)
    B200_AR(2);
  else if (vpt <= 4)
    B200_AR(4);
  else
    B200_AR(8);
#undef B200_AR
}

void run_fused_allreduce(const ArParams& a, cudaStream_t s) {
  B200_REQUIRE(a.world >= 2 && a.world <= kMaxRanks, "custom all-reduce: world size");
  B200_REQUIRE(a.H % 8 == 0 && a.H / 8 <= 1024 * 8, "custom all-reduce: hidden size");
  B200_REQUIRE(a.blocks >= 1 && a.blocks <= kMaxBlocks, "custom all-reduce: block count");
  B200_REQUIRE(a.rs_rows == 0 || (a.two_shot && a.rs_rows == (a.T + a.world - 1) / a.world),
               "custom all-reduce: epilogue reduce-scatter needs two-shot with ceil(T/world) rows");
  if (a.T == 0) return;
  const int nvec = a.H / 8;
  int threads = 128;
  while (threads < 512 && (nvec + threads - 1) / threads > 2) threads *= 2;
  const int vpt = (nvec + threads - 1) / threads;
  B200_REQUIRE(vpt <= 8, "custom all-reduce: hidden size too large");
  const bool norm = a.weight != nullptr;
  // warp-per-row kernel once blocks would walk several rows (one-shot: measured 25.4 us vs 22.2
  // us for the block kernel at 256 rows, TP=2, so it takes over beyond two rows per block)
  const int rows_per_rank = a.two_shot ? (a.T + a.world - 1) / a.world : a.T;
  if (rows_per_rank > (a.two_shot ? 1 : 2) * a.blocks && nvec <= 32 * 16 &&  // rows in registers
      (a.world == 2 || a.world == 4 || a.world == 8)) {
    // several rows per block: warp-per-row kernel keeps them all in flight
    if (a.two_shot) {
      if (norm)
        dispatch_warp_rows<true, true>(a, nvec, s);
      else
        dispatch_warp_rows<false, true>(a, nvec, s);
    } else {
      if (norm)
        dispatch_warp_rows<true, false>(a, nvec, s);
      else
        dispatch_warp_rows<false, false>(a, nvec, s);
    }
  } else if (a.two_shot) {
    if (norm)
      launch<true, true>(a, threads, vpt, a.blocks, s);
    else
      launch<false, true>(a, threads, vpt, a.blocks, s);
  } else {
    if (norm)
      launch<true, false>(a, threads, vpt, a.blocks, s);
    else
      launch<false, false>(a, threads, vpt, a.blocks, s);
  }
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

// ------------------------------------------------------------------------------ sampling
__global__ void __launch_bounds__(256) cand_exchange_kernel(CandParams a) {
  __shared__ uint32_t epoch_s;
  __shared__ int ok_all;
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < a.R) {
    for (int p = 0; p < a.world; ++p) {
      a.vals[p][(size_t)a.rank * a.R + r] = a.my_vals[r];
      a.ids[p][(size_t)a.rank * a.R + r] = a.my_ids[r];
    }
  }
  __threadfence_system();
  if (threadIdx.x == 0) {
    epoch_s = a.epochs[blockIdx.x] + 1;
    a.epochs[blockIdx.x] = epoch_s;
    ok_all = 1;
  }
  __syncthreads();
  const uint32_t epoch = epoch_s;
  if (threadIdx.x < a.world) {
    const int p = threadIdx.x;
    const size_t phase = 4 + a.parity;
    uint32_t* peer_slot = a.flags[p] + (phase * kMaxBlocks + blockIdx.x) * kMaxRanks + a.rank;
    st_release_sys(peer_slot, epoch);
    const uint32_t* my_slot = a.flags[a.rank] + (phase * kMaxBlocks + blockIdx.x) * kMaxRanks + p;
    const long long t0 = clock64();
    for (uint32_t spin = 1; (int32_t)(ld_acquire_sys(my_slot) - epoch) < 0; ++spin) {
      if ((spin & 31) != 0) continue;  // error word / clock every 32nd poll
      if (clock64() - t0 > kWaitBudgetCycles) {
        record_error(a.err, kErrPeerTimeout);
        ok_all = 0;
        break;
      }
      if (error_raised(a.err)) {
        ok_all = 0;
        break;
      }
    }
  }
  __syncthreads();
  if (!ok_all || r >= a.R) return;
  float bv = -INFINITY;
  int64_t bi = a.my_ids[r];
  for (int p = 0; p < a.world; ++p) {
    const float v = a.vals[a.rank][(size_t)p * a.R + r];
    const int64_t i = a.ids[a.rank][(size_t)p * a.R + r];
    if (v > bv || (v == bv && i < bi)) {
      bv = v;
      bi = i;
    }
  }
  a.out[r] = bi;
}

void run_exchange_candidates(const CandParams& a, cudaStream_t s) {
  B200_REQUIRE(a.world >= 2 && a.world <= kMaxRanks, "candidate exchange: world size");
  if (a.R == 0) return;
  const int blocks = (a.R + 255) / 256;
  B200_REQUIRE(blocks <= kMaxBlocks, "candidate exchange: too many rows");
  cand_exchange_kernel<<<blocks, 256, 0, s>>>(a);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

// ------------------------------------------------------------------------------ IPC helpers
void* ipc_malloc(size_t bytes) {
  void* p = nullptr;
  B200_CUDA_OK(cudaMalloc(&p, bytes));
  B200_CUDA_OK(cudaMemset(p, 0, bytes));
  return p;
}
void ipc_free(void* p) { B200_CUDA_OK(cudaFree(p)); }
std::string ipc_handle(void* p) {
  cudaIpcMemHandle_t h;
  B200_CUDA_OK(cudaIpcGetMemHandle(&h, p));
  return std::string(reinterpret_cast<const char*>(&h), sizeof(h));
}
void* ipc_open(const std::string& handle) {
  B200_REQUIRE(handle.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  B200_CUDA_OK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return p;
}
void ipc_close(void* p) { B200_CUDA_OK(cudaIpcCloseMemHandle(p)); }

}  // namespace comm
}  // namespace b200
