// NVLS (NVLink SHARP) all-reduce fused with residual-add + RMSNorm (+ optional per-token
// 1x128 e4m3 quantisation), for tensor parallelism over NVSwitch.
//
// Every rank's communicator buffer is bound to one NVLink multicast object (set up by the
// host through PyTorch's symmetric memory), so each buffer offset has two addresses: the
// rank's own copy (a plain device pointer) and a multicast address.  Through the multicast
// address the switch does the collective work:
//   multimem.ld_reduce  one 16-byte load returns the element-wise sum of the 16 bytes at
//                       that offset over every rank's copy (the switch reads all copies and
//                       adds them, accumulating in fp32);
//   multimem.st         one store writes every rank's copy;
//   multimem.red        one atomic add lands in every rank's copy (barrier counters).
//
//  two-shot (reduce-scatter + all-gather, the large-message algorithm): start barrier; rank r
//     reduces only its row chunk with multimem.ld_reduce, adds the residual rows it owns (the
//     residual stream stays row-sharded, as in the peer-to-peer two-shot kernel), normalises,
//     and multimem.st's the normalised row (or its e4m3 bytes and group scales) once, which
//     delivers it to every rank; end barrier.  Each rank's NVLink carries about one copy of
//     the message in each direction, against (2 - 2/world) copies for the peer-to-peer
//     two-shot.
//  one-shot (small messages): start barrier; every rank reduces all rows with
//     multimem.ld_reduce and writes its own output copy with plain stores; no end barrier.
//
// Barriers are per block and use monotonic counters in the multicast buffer: block b of every
// rank adds 1 to counter[phase][b] of every rank with one multimem.red (release, system
// scope), then spins with acquire loads on its own copy until the counter reaches
// epoch * world, where epoch is this block's local call count for that phase.  A rank can run
// at most one call ahead of the slowest (it must pass the next start barrier), and the two
// buffer parities alternate, so the counters never need resetting.  Every spin is bounded by
// a clock budget; on expiry the kernel records kErrPeerTimeout and returns.
//
// No TMA is used here; loads and stores through the multicast address are the multimem
// instructions above (open on any number of GPUs).  Reference counterpart: the peer-to-peer
// fused all-reduce of vllm_musa/jit_kernel/csrc/distributed/custom_all_reduce.mu:847-1126;
// the NVLS algorithm is this build's Blackwell / NVSwitch upgrade of it.
#include <algorithm>

#include "../b200_kernels.h"
#include "../common/common.cuh"
#include "custom_ar.h"

namespace b200 {
namespace comm {

namespace {

B200_DEVICE uint4 mm_ld_reduce_bf16x8(const void* mc) {
  uint4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(mc)
               : "memory");
  return r;
}

B200_DEVICE void mm_st_16(void* mc, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

B200_DEVICE void mm_st_8(void* mc, uint32_t a, uint32_t b) {
  asm volatile("multimem.st.relaxed.sys.global.v2.f32 [%0], {%1, %2};" ::"l"(mc), "r"(a), "r"(b)
               : "memory");
}

B200_DEVICE void mm_st_f32(void* mc, float v) {
  asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(mc), "f"(v) : "memory");
}

B200_DEVICE void mm_red_add_release(uint32_t* mc, uint32_t v) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(mc), "r"(v) : "memory");
}

B200_DEVICE uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Block barrier among the ranks through the multicast counter of (phase, block).  Called by
// every thread of the block; returns false on timeout (error recorded).
B200_DEVICE bool nvls_barrier(const NvlsParams& a, int phase, uint32_t epoch) {
  __shared__ int ok_all;
  __syncthreads();  // every thread's prior stores (incl. multimem.st) precede the release
  if (threadIdx.x == 0) {
    ok_all = 1;
    const size_t idx = (size_t)phase * kMaxBlocks + blockIdx.x;
    __threadfence_system();
    mm_red_add_release(a.mc_flags + idx, 1u);
    const uint32_t target = epoch * (uint32_t)a.world;
    const long long t0 = clock64();
    for (uint32_t spin = 1; (int32_t)(ld_acquire_sys_u32(a.flags + idx) - target) < 0; ++spin) {
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

// Quantise 8 values (this lane's vector of a 128-element group shared by 16 lanes) to e4m3;
// returns the group scale (amax / 448, as group_quant_fp8_kernel) and the packed bytes.
B200_DEVICE float quant8(const float (&f)[8], uint32_t& lo, uint32_t& hi) {
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(f[j]));
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = fmaxf(amax, 1e-10f) / 448.f;
  const float inv = 1.f / scale;
  uint8_t b[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const __nv_fp8_e4m3 q(f[j] * inv);
    b[j] = *reinterpret_cast<const uint8_t*>(&q);
  }
  lo = (uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) | ((uint32_t)b[3] << 24);
  hi = (uint32_t)b[4] | ((uint32_t)b[5] << 8) | ((uint32_t)b[6] << 16) | ((uint32_t)b[7] << 24);
  return scale;
}

constexpr int kNvlsThreads = 256;
constexpr int kNvlsWarps = kNvlsThreads / 32;

// This lane's VPW vectors of `row`, summed over the ranks by the switch.
template <int VPW>
B200_DEVICE void load_row(const NvlsParams& a, int row, int lane, int nvec, uint4 (&v)[VPW]) {
  const char* src = reinterpret_cast<const char*>(a.mc_staging) + (size_t)row * a.H * 2;
#pragma unroll
  for (int i = 0; i < VPW; ++i) {
    const int c = lane + 32 * i;
    if (c < nvec) v[i] = mm_ld_reduce_bf16x8(src + (size_t)c * 16);
  }
}

// Residual add, RMSNorm, optional e4m3 quantisation and the store (multicast for two-shot,
// local for one-shot) of one reduced row.
template <int VPW, bool kNorm, bool kTwoShot, bool kQuant>
B200_DEVICE void finish_row(const NvlsParams& a, int row, int lane, int nvec, uint4 (&packed)[VPW]) {
  const size_t row_bytes = (size_t)a.H * 2;
  if (a.residual) {
    uint4* rr = reinterpret_cast<uint4*>(reinterpret_cast<char*>(a.residual) + row * row_bytes);
#pragma unroll
    for (int i = 0; i < VPW; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
        float v[8], r[8];
        unpack8(packed[i], v);
        unpack8(rr[c], r);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] += r[j];
        packed[i] = pack8(v);
        rr[c] = packed[i];
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
    // a 128-element group is 16 consecutive vectors = 16 lanes of one i: all 32 lanes take
    // part in the group reduction, so the bound check is uniform per i (nvec % 32 == 0 when
    // quantising)
    if (!kQuant && c >= nvec) continue;
    if (kQuant && 32 * i >= nvec) continue;
    float f[8];
    unpack8(packed[i], f);
    if constexpr (kNorm) {
      float w[8];
      unpack8(reinterpret_cast<const uint4*>(a.weight)[c], w);
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = f[j] * inv * w[j];
    }
    if constexpr (kQuant) {
      // bf16 rounding first, as the unfused path quantises the bf16 normalised row
      const uint4 ov = pack8(f);
      unpack8(ov, f);
      uint32_t lo, hi;
      const float scale = quant8(f, lo, hi);
      const size_t qoff = (size_t)row * a.H + (size_t)c * 8;
      const size_t soff = (size_t)row * (a.H / 128) + c / 16;
      if (kTwoShot) {
        mm_st_8(reinterpret_cast<char*>(a.mc_q) + qoff, lo, hi);
        if ((lane & 15) == 0) mm_st_f32(reinterpret_cast<char*>(a.mc_s) + soff * 4, scale);
      } else {
        *reinterpret_cast<uint2*>(reinterpret_cast<char*>(a.q_local) + qoff) = make_uint2(lo, hi);
        if ((lane & 15) == 0) a.s_local[soff] = scale;
      }
    } else {
      const uint4 ov = pack8(f);
      if (kTwoShot)
        mm_st_16(reinterpret_cast<char*>(a.mc_out) + row * row_bytes + (size_t)c * 16, ov);
      else
        reinterpret_cast<uint4*>(reinterpret_cast<char*>(a.out_local) + row * row_bytes)[c] = ov;
    }
  }
}

// One warp per row; lane l owns the 16-byte vectors l, l + 32, ... (VPW of them).  A warp that
// walks several rows (beyond the block cap) issues the next row's multimem.ld_reduce before it
// finishes and stores the current one (rows up to 16 vectors per lane).
template <int VPW, bool kNorm, bool kTwoShot, bool kQuant>
__global__ void __launch_bounds__(kNvlsThreads) nvls_ar_kernel(NvlsParams a) {
  constexpr bool kPipe = VPW <= 16;
  __shared__ uint32_t epoch_s[2];
  if (threadIdx.x == 0) {
    epoch_s[0] = a.epochs[blockIdx.x] + 1;
    a.epochs[blockIdx.x] = epoch_s[0];
    if (kTwoShot) {
      epoch_s[1] = a.epochs[kMaxBlocks + blockIdx.x] + 1;
      a.epochs[kMaxBlocks + blockIdx.x] = epoch_s[1];
    }
  }
  __syncthreads();
  if (!nvls_barrier(a, 0, epoch_s[0])) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvec = a.H / 8;
  const int per = kTwoShot ? (a.T + a.world - 1) / a.world : a.T;
  const int r0 = kTwoShot ? min(a.T, a.rank * per) : 0, r1 = min(a.T, r0 + per);
  const int stride = gridDim.x * kNvlsWarps;
  int row = r0 + blockIdx.x * kNvlsWarps + warp;
  uint4 cur[VPW];
  if (row < r1) load_row<VPW>(a, row, lane, nvec, cur);
  while (row < r1) {
    const int next = row + stride;
    if constexpr (kPipe) {
      uint4 nxt[VPW];
      if (next < r1) load_row<VPW>(a, next, lane, nvec, nxt);
      finish_row<VPW, kNorm, kTwoShot, kQuant>(a, row, lane, nvec, cur);
#pragma unroll
      for (int i = 0; i < VPW; ++i) cur[i] = nxt[i];
    } else {
      finish_row<VPW, kNorm, kTwoShot, kQuant>(a, row, lane, nvec, cur);
      if (next < r1) load_row<VPW>(a, next, lane, nvec, cur);
    }
    row = next;
  }
  if (kTwoShot) nvls_barrier(a, 1, epoch_s[1]);
}

template <int VPW, bool kNorm, bool kTwoShot>
void launch_q(const NvlsParams& a, cudaStream_t s) {
  if (a.mc_q != nullptr || a.q_local != nullptr)
    nvls_ar_kernel<VPW, kNorm, kTwoShot, true><<<a.blocks, kNvlsThreads, 0, s>>>(a);
  else
    nvls_ar_kernel<VPW, kNorm, kTwoShot, false><<<a.blocks, kNvlsThreads, 0, s>>>(a);
}

template <int VPW, bool kNorm>
void launch_shot(const NvlsParams& a, cudaStream_t s) {
  if (a.two_shot)
    launch_q<VPW, kNorm, true>(a, s);
  else
    launch_q<VPW, kNorm, false>(a, s);
}

template <int VPW>
void launch_norm(const NvlsParams& a, cudaStream_t s) {
  if (a.weight != nullptr)
    launch_shot<VPW, true>(a, s);
  else
    launch_shot<VPW, false>(a, s);
}

}  // namespace

int nvls_blocks(int T, int world, bool two_shot, int rows_per_warp) {
  const int rows = two_shot ? (T + world - 1) / world : T;
  // one row per warp up to the block cap (measured at TP=2, 1024 / 4096 / 8192 rows: 42.9 /
  // 120.6 / 207.5 us with one row per warp, 46.0 / 121.0 / 207.6 with two, 58.1 / 112.6 /
  // 207.6 with four: the multicast reduce is not phase-bound at these sizes)
  const int rpw = rows_per_warp > 0 ? rows_per_warp : 1;
  const int blocks = (rows + kNvlsWarps * rpw - 1) / (kNvlsWarps * rpw);
  return std::max(1, std::min(kMaxBlocks, blocks));
}

void run_nvls_allreduce(const NvlsParams& a, cudaStream_t s) {
  B200_REQUIRE(a.world >= 2 && a.world <= kMaxRanks, "nvls all-reduce: world size");
  B200_REQUIRE(a.H % 8 == 0 && a.H / 8 <= 32 * 32, "nvls all-reduce: hidden size (<= 8192)");
  B200_REQUIRE(a.blocks >= 1 && a.blocks <= kMaxBlocks, "nvls all-reduce: block count");
  B200_REQUIRE(a.mc_staging && a.mc_flags && a.flags && a.epochs, "nvls all-reduce: buffers");
  B200_REQUIRE(a.two_shot ? a.mc_out != nullptr || a.mc_q != nullptr
                          : a.out_local != nullptr || a.q_local != nullptr,
               "nvls all-reduce: output");
  const bool quant = a.mc_q != nullptr || a.q_local != nullptr;
  B200_REQUIRE(!quant || (a.H % 256 == 0 && a.weight != nullptr),
               "nvls all-reduce: the fp8 output needs a normalised row of a multiple of 256");
  if (a.T == 0) return;
  const int nvec = a.H / 8;
  if (nvec <= 32 * 4)
    launch_norm<4>(a, s);
  else if (nvec <= 32 * 8)
    launch_norm<8>(a, s);
  else if (nvec <= 32 * 16)
    launch_norm<16>(a, s);
  else
    launch_norm<32>(a, s);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

}  // namespace comm
}  // namespace b200
