// Block-scaled FP8 (e4m3) GEMM on the sm_100a tensor cores (DeepSeek-style quantisation).
//
//   C[M, N] (bf16) = sum_kb  sa[m, kb] * sb[n / 128, kb] * (A[m, kb] . B[n, kb]^T)
//
// A = activations quantised per token in 1 x 128 groups (fp32 scales sa [M, K/128]), B = a
// weight quantised in 128 x 128 blocks (fp32 scales sb [N/128, K/128]), kb = 128-wide K block.
// The scales change every K block, so the fp32 partial product of each K block must be scaled
// before it joins the sum.  Blackwell's tcgen05 accumulates in TMEM, so the kernel keeps a ring
// of per-K-block partial tiles there:
//
//   warp 0      TMA producer: per K block a 128 x 128-byte A tile and a 128 x 128-byte B tile
//               (128-byte swizzle) into a ring of shared-memory stages.
//   warp 1      allocates TMEM (4 slots x 128 columns); one lane issues 4 tcgen05.mma
//               kind::f8f6f4 (M=128, N=128, K=32) per K block into a fresh slot and commits.
//   warps 2..9  epilogue ("promotion"): tcgen05.ld the slot, multiply by sa*sb, add into fp32
//               registers (each warp owns 32 rows x 64 columns), release the slot; after the
//               last K block of the unit write bf16 (or split-K fp32 partials, summed in-kernel
//               by the last-arriving CTA of the tile).
//
// The MMA of K block kb+1..kb+3 overlaps the promotion of K block kb.  Reference counterparts:
// vllm_musa/model_executor/layers/quantization/kernels/linear/scaled_mm/deep_gemm.py:92-198
// (DeepGEMM fp8_gemm_nt, no source in the reference) and vllm_musa/kernels/fp8_block_gemm.py:18,
// fp8_block_splitk.py:85-147 (Triton block-scaled GEMM and split-K).
#include <algorithm>

#include "../b200_kernels.h"
#include "../common/common.cuh"
#include "../common/tcgen05.cuh"
#include "../common/tma_host.h"

namespace b200 {
namespace gemm_fp8 {

constexpr int BM = 128, BN = 128, BK = 128;  // BK in e4m3 elements = one 128-byte swizzle atom
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kSlots = 4;  // TMEM ring of per-K-block partial tiles
constexpr int kStageBytes = (BM + BN) * BK;
constexpr int kMaxStages = 6;
constexpr int kSmemBytes = kMaxStages * kStageBytes + 1024 + 512;
constexpr int kGroupN = 8;

struct Params {
  int M, N, K;
  int num_m, num_n, num_kb, splits, kb_per_split, total_units;
  const float* sa;
  int64_t sa_ld;  // row stride of sa (>= num_kb)
  const float* sb;
  int64_t sb_ld;  // row stride of sb (>= num_kb)
  __nv_bfloat16* C;
  int64_t ldc;
  float* ws;      // split-K partials [splits, M, N]
  int* counters;  // one per output tile, zero between launches
  int* err;
  // grouped (MoE) mode: m-tile i multiplies expert tile_expert[i] (B rows e*N.., scale rows
  // e*ceil(N/128)..); the live m-tile count is read from the device
  const int32_t* tile_expert;
  const int32_t* num_tiles;
};

B200_DEVICE void epi_barrier() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
B200_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
B200_DEVICE void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

B200_DEVICE void unit_coords(int u, const Params& p, int& m, int& n, int& ks) {
  const int tiles = p.num_m * p.num_n;
  ks = u / tiles;
  const int t = u - ks * tiles;
  const int group = kGroupN * p.num_m;
  const int g = t / group;
  const int r = t - g * group;
  const int n0 = g * kGroupN;
  const int gn = min(kGroupN, p.num_n - n0);
  m = r / gn;
  n = n0 + (r - m * gn);
}

B200_DEVICE void store_row64(const Params& p, int row, int col0, const float (&f)[64]) {
  __nv_bfloat16* C = p.C + (size_t)row * p.ldc + col0;
#pragma unroll
  for (int v = 0; v < 8; ++v) {
    if (col0 + 8 * v < p.N) {
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = f[8 * v + j];
      *reinterpret_cast<uint4*>(C + 8 * v) = pack8(o);
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    Params p, int stages) {
  pdl_trigger();
  if (p.tile_expert) {
    pdl_wait();  // the live tile count comes from the preceding alignment kernel
    p.num_m = *p.num_tiles;
    p.total_units = p.num_m * p.num_n;
  }
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kMaxStages * kStageBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + kMaxStages;
  uint64_t* slot_full = bars + 2 * kMaxStages;
  uint64_t* slot_empty = slot_full + kSlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(slot_empty + kSlots);
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&slot_full[s], 1);
      mbar_init(&slot_empty[s], kEpiWarps);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, kSlots * BN);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      pdl_wait();
      for (int u = blockIdx.x; u < p.total_units && ok; u += gridDim.x) {
        int m, n, ks;
        unit_coords(u, p, m, n, ks);
        const int kb0 = ks * p.kb_per_split;
        const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + stage * kStageBytes;
          mbar_arrive_expect_tx(&full[stage], kStageBytes);
          tma_load_2d(st, &tmA, &full[stage], kb * BK, m * BM);
          const int brow = p.tile_expert ? p.tile_expert[m] * p.N + n * BN : n * BN;
          tma_load_2d(st + BM * BK, &tmB, &full[stage], kb * BK, brow);
          if (++stage == stages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (ok) {  // drain: no TMA write may be in flight when the CTA exits
        for (int i = 0; i < stages; ++i) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err)) break;
          if (++stage == stages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_e4m3(BM, BN);
      int stage = 0, slot = 0;
      uint32_t phase = 0, slot_phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < p.total_units && ok; u += gridDim.x) {
        int m, n, ks;
        unit_coords(u, p, m, n, ks);
        const int kb0 = ks * p.kb_per_split;
        const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&slot_empty[slot], slot_phase ^ 1, p.err) ||
              !mbar_wait(&full[stage], phase, p.err)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint32_t sa = smem_u32(smem + stage * kStageBytes);
          const uint64_t adesc = tc::smem_desc_kmajor_sw128(sa);
          const uint64_t bdesc = tc::smem_desc_kmajor_sw128(sa + BM * BK);
          const uint32_t d = tmem_base + slot * BN;
#pragma unroll
          for (int k = 0; k < BK / 32; ++k)  // +32 bytes along K -> +2 in the >>4 address field
            tc::mma_f8f6f4_ss(d, adesc + 2 * k, bdesc + 2 * k, idesc, k > 0 ? 1u : 0u);
          tc::mma_commit(&empty[stage]);
          tc::mma_commit(&slot_full[slot]);
          if (++stage == stages) {
            stage = 0;
            phase ^= 1;
          }
          if (++slot == kSlots) {
            slot = 0;
            slot_phase ^= 1;
          }
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- promotion epilogue
    const int q = warp & 3;               // TMEM lane quarter (rows q*32 .. q*32+31)
    const int half = (warp - 2) >> 2;     // column half of the 128-wide tile
    const bool split = p.splits > 1;
    int slot = 0;
    uint32_t slot_phase = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < p.total_units && ok; u += gridDim.x) {
      int m, n, ks;
      unit_coords(u, p, m, n, ks);
      const int kb0 = ks * p.kb_per_split;
      const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
      const int row = m * BM + q * 32 + lane;
      const bool row_ok = row < p.M;
      const float* sa_row = p.sa + (size_t)(row_ok ? row : 0) * p.sa_ld;
      const int nb = p.tile_expert ? p.tile_expert[m] * ((p.N + BN - 1) / BN) + n : n;
      const float* sb_row = p.sb + (size_t)nb * p.sb_ld;
      float acc[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) acc[j] = 0.f;
      float scale_next = row_ok ? __ldg(sa_row + kb0) * __ldg(sb_row + kb0) : 0.f;
      for (int kb = kb0; kb < kb1; ++kb) {
        const float scale = scale_next;
        if (kb + 1 < kb1)
          scale_next = row_ok ? __ldg(sa_row + kb + 1) * __ldg(sb_row + kb + 1) : 0.f;
        if (!mbar_wait(&slot_full[slot], slot_phase, p.err)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const uint32_t t = tmem_base + ((uint32_t)(q * 32) << 16) + slot * BN + half * 64;
        uint32_t r0[32], r1[32];
        tc::tmem_ld_32x32b_x32(t, r0);
        tc::tmem_ld_32x32b_x32(t + 32, r1);
        tc::tmem_ld_wait();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&slot_empty[slot]);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          acc[j] = fmaf(scale, __uint_as_float(r0[j]), acc[j]);
          acc[32 + j] = fmaf(scale, __uint_as_float(r1[j]), acc[32 + j]);
        }
        if (++slot == kSlots) {
          slot = 0;
          slot_phase ^= 1;
        }
      }
      if (!ok) break;
      const int col0 = n * BN + half * 64;
      if (!split) {
        if (row_ok) store_row64(p, row, col0, acc);
        continue;
      }
      if (row_ok) {
        float* w = p.ws + ((size_t)ks * p.M + row) * p.N + col0;
#pragma unroll
        for (int v = 0; v < 16; ++v)
          if (col0 + 4 * v < p.N)
            reinterpret_cast<float4*>(w)[v] =
                make_float4(acc[4 * v], acc[4 * v + 1], acc[4 * v + 2], acc[4 * v + 3]);
      }
      __threadfence();
      epi_barrier();
      const int tile = m * p.num_n + n;
      if (warp == 2 && lane == 0) s_last = atomicAdd(&p.counters[tile], 1) == p.splits - 1;
      epi_barrier();
      if (s_last) {
        __threadfence();
        if (row_ok) {
          float f[64];
#pragma unroll
          for (int j = 0; j < 64; ++j) f[j] = 0.f;
          for (int sp = 0; sp < p.splits; ++sp) {
            const float4* w =
                reinterpret_cast<const float4*>(p.ws + ((size_t)sp * p.M + row) * p.N + col0);
#pragma unroll
            for (int v = 0; v < 16; ++v) {
              if (col0 + 4 * v >= p.N) break;
              const float4 x = __ldcg(w + v);
              f[4 * v] += x.x;
              f[4 * v + 1] += x.y;
              f[4 * v + 2] += x.z;
              f[4 * v + 3] += x.w;
            }
          }
          store_row64(p, row, col0, f);
        }
        epi_barrier();
        if (warp == 2 && lane == 0) p.counters[tile] = 0;
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 1) tc::tmem_dealloc(tmem_base, kSlots * BN);
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------
Fp8Plan plan_fp8(int M, int N, int K) {
  const int sms = num_sms();
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int num_kb = (K + BK - 1) / BK;
  int s = 1;
  // split K while fewer than ~half the SMs have a tile and every split keeps >= 4 K blocks
  while (tiles * s * 2 <= sms && num_kb / (s * 2) >= 4 && (long)(s * 2) * M * N <= (32l << 20))
    s *= 2;
  const int kps = (num_kb + s - 1) / s;
  s = (num_kb + kps - 1) / kps;
  Fp8Plan p;
  p.splits = s;
  p.workspace_floats = s > 1 ? (long)s * M * N : 0;
  p.counters = s > 1 ? tiles : 0;
  return p;
}

void run_fp8(const Fp8GemmArgs& a, cudaStream_t stream) {
  const int M = a.M, N = a.N, K = a.K;
  B200_REQUIRE(K % 16 == 0 && N % 16 == 0, "gemm_fp8: K and N must be multiples of 16");
  if (M == 0) return;
  Params p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.num_m = (M + BM - 1) / BM;
  p.num_n = (N + BN - 1) / BN;
  p.num_kb = (K + BK - 1) / BK;
  int s = a.tile_expert ? 1
          : a.splits > 0 ? std::min(a.splits, p.num_kb)
                         : plan_fp8(M, N, K).splits;
  p.kb_per_split = (p.num_kb + s - 1) / s;
  s = (p.num_kb + p.kb_per_split - 1) / p.kb_per_split;
  p.splits = s;
  p.total_units = p.num_m * p.num_n * s;
  p.sa = a.sa;
  p.sa_ld = a.sa_ld;
  p.sb = a.sb;
  p.sb_ld = a.sb_ld;
  p.C = reinterpret_cast<__nv_bfloat16*>(a.C);
  p.ldc = a.ldc;
  p.err = a.err;
  p.ws = a.workspace;
  p.counters = a.counters;
  p.tile_expert = a.tile_expert;
  p.num_tiles = a.num_tiles;
  if (a.tile_expert) {
    B200_REQUIRE(s == 1 && a.num_tiles && M % BM == 0 && a.num_experts > 0,
                 "gemm_fp8 grouped: no split-K, rows a multiple of 128");
  }
  if (s > 1) {
    B200_REQUIRE(a.workspace && a.workspace_numel >= (long)s * M * N,
                 "gemm_fp8: split-K workspace too small");
    B200_REQUIRE(a.counters && a.counters_numel >= p.num_m * p.num_n,
                 "gemm_fp8: split-K counters too small");
  }
  const CUtensorMap ta = make_tma_2d(const_cast<void*>(a.A), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K,
                                     M, a.lda, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tb =
      make_tma_2d(const_cast<void*>(a.B), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K,
                  (uint64_t)(a.tile_expert ? a.num_experts : 1) * N, a.ldb, BK, BN,
                  CU_TENSOR_MAP_SWIZZLE_128B);
  const int stages = kMaxStages;
  ensure_dynamic_smem(reinterpret_cast<const void*>(gemm_fp8_kernel), kSmemBytes);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(std::min(p.total_units, num_sms()));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B200_CUDA_OK(cudaLaunchKernelEx(&cfg, gemm_fp8_kernel, ta, tb, p, stages));
  count_launch();
}

}  // namespace gemm_fp8
}  // namespace b200
