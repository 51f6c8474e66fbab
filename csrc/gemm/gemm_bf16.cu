// Persistent BF16 GEMM on the sm_100a 5th-generation tensor cores.
//
//   C[M, N] = A[M, K] . B[N, K]^T        (A = activations, B = nn.Linear weight, both K-major)
//
// Replaces the vendor BF16 GEMM the reference routes unquantized linears to
// (reference: setup.py:258 links mublasLt; vllm_musa/kernels/fp8_block_gemm.py:18 is its
// Triton GEMM) with a hand-written tcgen05 kernel:
//
//   warp 0      TMA producer: 128x64 A tile + BNx64 B tile per stage (128B swizzle), ring of
//               STAGES shared-memory slots guarded by full/empty mbarriers.
//   warp 1      allocates TMEM (2 x BN fp32 columns: double-buffered accumulators), one
//               elected lane issues tcgen05.mma (M=128, N=BN, K=16) and tcgen05.commit.
//   warps 2..5  epilogue: tcgen05.ld accumulator rows -> fused epilogue -> global.
//
// Work units (m-tile, n-tile, k-split) are scheduled persistently (grid <= #SMs) in grouped
// order so that a wave shares B tiles through L2.  Epilogues:
//   kStore     C = acc (bf16)
//   kSiluMul   B rows are interleaved in groups of 64 (32 gate rows, 32 up rows); output
//              C[:, g*32 + c] = silu(acc[g*64 + c]) * acc[g*64 + 32 + c]  (N/2 columns)
//   kF32       C = acc (fp32, used for logits)
//   kSplitK    partial sums to an fp32 workspace [splits, M, N]; a reduce kernel finishes.
// Every mbarrier wait is bounded (see common.cuh); a timeout leaves an error code and the
// kernel drains, frees TMEM and returns.
#include <algorithm>
#include <vector>

#include "../b200_kernels.h"
#include "../common/common.cuh"
#include "../common/tcgen05.cuh"
#include "../common/tma_host.h"

namespace b200 {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle atom
constexpr int kThreads = 192;
constexpr int kGroupN = 8;

enum Epilogue : int { kStore = 0, kSiluMul = 1, kF32 = 2, kSplitK = 3 };

struct Params {
  int M, N, K;
  int num_m, num_n, num_kb, splits, kb_per_split;
  int total_units;
  void* C;       // output (bf16 or fp32) or fp32 workspace for split-K
  int ldc;       // elements
  int* err;
};

template <int BN>
struct Smem {
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (BN == 256) ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int kBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

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

B200_DEVICE float silu(float x) { return x / (1.f + __expf(-x)); }

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB, Params p) {
  using S = Smem<BN>;
  constexpr int STAGES = S::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::kABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * S::kStageBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = bars + 2 * STAGES + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);  // one arrive per epilogue warp
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, 2 * BN);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
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
          mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
          tma_load_2d(sA + stage * S::kABytes, &tmA, &full[stage], kb * BK, m * BM);
          tma_load_2d(sB + stage * S::kBBytes, &tmB, &full[stage], kb * BK, n * BN);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: wait until the MMA warp has released every slot we filled, so no TMA write
      // is in flight when the CTA exits.
      if (ok) {
        for (int i = 0; i < STAGES; ++i) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err)) break;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_f16<true>(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < p.total_units && ok; u += gridDim.x) {
        int m, n, ks;
        unit_coords(u, p, m, n, ks);
        const int kb0 = ks * p.kb_per_split;
        const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, p.err)) break;
        tc::fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint64_t adesc = tc::smem_desc_kmajor_sw128(smem_u32(sA + stage * S::kABytes));
          const uint64_t bdesc = tc::smem_desc_kmajor_sw128(smem_u32(sB + stage * S::kBBytes));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // +32 bytes along K inside the 128-byte swizzle atom -> +2 in the >>4 address field
            tc::mma_f16_ss(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc,
                           (kb > kb0 || k > 0) ? 1u : 0u);
          }
          tc::mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc::mma_commit(&acc_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = blockIdx.x; u < p.total_units; u += gridDim.x) {
      int m, n, ks;
      unit_coords(u, p, m, n, ks);
      if (!mbar_wait(&acc_full[acc], acc_phase, p.err)) break;
      tc::fence_after_sync();
      const int row = m * BM + row_in_tile;
      const bool row_ok = row < p.M;
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
      if constexpr (EPI == kSiluMul) {
        __nv_bfloat16* C = reinterpret_cast<__nv_bfloat16*>(p.C);
#pragma unroll 1
        for (int g = 0; g < BN / 64; ++g) {
          uint32_t rg[32], ru[32];
          tc::tmem_ld_32x32b_x32(t_row + g * 64, rg);
          tc::tmem_ld_32x32b_x32(t_row + g * 64 + 32, ru);
          tc::tmem_ld_wait();
          const int col = (n * BN + g * 64) / 2;  // output column base
          if (row_ok && col < p.N / 2) {
            uint4* dst = reinterpret_cast<uint4*>(C + (size_t)row * p.ldc + col);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              float f[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const float gv = __uint_as_float(rg[v * 8 + j]);
                const float uv = __uint_as_float(ru[v * 8 + j]);
                f[j] = silu(gv) * uv;
              }
              dst[v] = pack8(f);
            }
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tc::tmem_ld_32x32b_x32(t_row + c * 32, r);
          tc::tmem_ld_wait();
          const int col = n * BN + c * 32;
          if (!row_ok || col >= p.N) continue;
          if constexpr (EPI == kStore) {
            __nv_bfloat16* C = reinterpret_cast<__nv_bfloat16*>(p.C);
            uint4* dst = reinterpret_cast<uint4*>(C + (size_t)row * p.ldc + col);
            const int nvec = min(4, (p.N - col) / 8);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              if (v < nvec) {
                float f[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) f[j] = __uint_as_float(r[v * 8 + j]);
                dst[v] = pack8(f);
              }
            }
          } else {
            float* C = reinterpret_cast<float*>(p.C);
            if constexpr (EPI == kSplitK) C += (size_t)ks * p.M * p.ldc;
            float4* dst = reinterpret_cast<float4*>(C + (size_t)row * p.ldc + col);
            const int nvec = min(8, (p.N - col) / 4);
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              if (v < nvec)
                dst[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                     __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
            }
          }
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 1) tc::tmem_dealloc(tmem_base, 2 * BN);
}

// Sum split-K partials [splits, M, N] fp32 -> bf16 C (or fp32 C).
template <bool kOutF32>
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, void* __restrict__ C, int M,
                                     int N, int ldc, int splits) {
  const size_t total4 = (size_t)M * N / 4;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total4;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t e = i * 4;
    const int row = e / N, col = e % N;
    float4 acc = reinterpret_cast<const float4*>(ws)[i];
    for (int s = 1; s < splits; ++s) {
      const float4 t = reinterpret_cast<const float4*>(ws + (size_t)s * M * N)[i];
      acc.x += t.x;
      acc.y += t.y;
      acc.z += t.z;
      acc.w += t.w;
    }
    if constexpr (kOutF32) {
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(C) + (size_t)row * ldc + col) = acc;
    } else {
      __nv_bfloat16* c = reinterpret_cast<__nv_bfloat16*>(C) + (size_t)row * ldc + col;
      uint2 v;
      v.x = pack_bf16x2(acc.x, acc.y);
      v.y = pack_bf16x2(acc.z, acc.w);
      *reinterpret_cast<uint2*>(c) = v;
    }
  }
}

template <bool kOutF32>
__global__ void splitk_reduce_silu_kernel(const float* __restrict__ ws, __nv_bfloat16* __restrict__ C,
                                          int M, int N, int ldc, int splits) {
  // N = interleaved width; output width N/2
  const size_t total = (size_t)M * (N / 2);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int row = i / (N / 2), oc = i % (N / 2);
    const int g = oc / 32, c = oc % 32;
    const int cg = g * 64 + c, cu = g * 64 + 32 + c;
    float gv = 0.f, uv = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float* w = ws + (size_t)s * M * N + (size_t)row * N;
      gv += w[cg];
      uv += w[cu];
    }
    C[(size_t)row * ldc + oc] = __float2bfloat16_rn(silu(gv) * uv);
  }
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------
struct Plan {
  int bn, splits;
};

// Cost model: per-CTA time of one k-block is max(load time, MMA time) at the per-SM share of
// HBM bandwidth / tensor throughput; total = waves * k-blocks-per-unit * per-kb time, plus the
// split-K workspace round trip.
static Plan choose_plan(int M, int N, int K) {
  const int sms = num_sms();
  const int num_m = (M + BM - 1) / BM;
  const int num_kb = (K + BK - 1) / BK;
  Plan best{256, 1};
  double best_cost = 1e30;
  const int bns[3] = {256, 128, 64};
  for (int bi = 0; bi < 3; ++bi) {
    const int bn = bns[bi];
    const int num_n = (N + bn - 1) / bn;
    const int tiles = num_m * num_n;
    for (int s = 1; s <= 16; ++s) {
      if (s > 1 && (num_kb + s - 1) / s < 4) break;
      const int kps = (num_kb + s - 1) / s;
      const long units = (long)tiles * s;
      const long waves = (units + sms - 1) / sms;
      const long active = std::min<long>(units, sms);
      const double bytes = (double)(BM + bn) * BK * 2;
      const double per_sm_bw = 6.5e12 / active * 0.9;
      const double mma_t = (double)BM * bn * BK * 2 / (1.4e15 / sms);
      const double reuse = active > 1 ? 0.5 : 1.0;  // neighbours share tiles through L2
      const double load_t = bytes * reuse / per_sm_bw;
      double cost = waves * kps * std::max(load_t, mma_t) + waves * 1.5e-6;
      if (s > 1) cost += (double)M * N * 4 * (s + 1) / 6.0e12 + 3e-6;
      if (cost < best_cost * 0.97) {
        best_cost = cost;
        best = {bn, s};
      }
    }
  }
  return best;
}

template <int BN, int EPI>
static void launch(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p,
                   cudaStream_t stream) {
  auto kern = gemm_bf16_kernel<BN, EPI>;
  const int smem = Smem<BN>::kBytes;
  static uint32_t attr_set = 0;  // bit per device
  int dev;
  B200_CUDA_OK(cudaGetDevice(&dev));
  if (!(attr_set & (1u << dev))) {
    B200_CUDA_OK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_set |= 1u << dev;
  }
  const int grid = std::min(p.total_units, num_sms());
  kern<<<grid, kThreads, smem, stream>>>(ta, tb, p);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

template <int EPI>
static void dispatch_bn(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const Params& p,
                        cudaStream_t s) {
  if (bn == 256)
    launch<256, EPI>(ta, tb, p, s);
  else if (bn == 128)
    launch<128, EPI>(ta, tb, p, s);
  else
    launch<64, EPI>(ta, tb, p, s);
}

GemmPlan plan_bf16(int M, int N, int K) {
  Plan p = choose_plan(M, N, K);
  const int num_kb = (K + BK - 1) / BK;
  int s = std::max(1, std::min<int>(p.splits, num_kb));
  const int kps = (num_kb + s - 1) / s;
  s = (num_kb + kps - 1) / kps;
  return GemmPlan{p.bn, s, s > 1 ? (int64_t)s * M * N : 0};
}

void run_bf16(const GemmArgs& a, cudaStream_t stream) {
  const int M = a.M, N = a.N, K = a.K;
  B200_REQUIRE(K % 8 == 0 && N % 8 == 0, "gemm_bf16: K and N must be multiples of 8");
  B200_REQUIRE((a.lda * 2) % 16 == 0 && (a.ldb * 2) % 16 == 0,
               "gemm_bf16: row strides must be 16-byte multiples");
  B200_REQUIRE(reinterpret_cast<uintptr_t>(a.A) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(a.B) % 16 == 0,
               "gemm_bf16: operands must be 16-byte aligned");
  if (M == 0) return;
  const bool silu = a.mode == kModeSiluMul;
  B200_REQUIRE(!silu || N % 64 == 0, "gemm_bf16 silu: N must be a multiple of 64");
  GemmPlan plan = plan_bf16(M, N, K);
  if (a.bn > 0) plan.bn = a.bn;
  if (a.splits > 0) plan.splits = a.splits;
  B200_REQUIRE(plan.bn == 64 || plan.bn == 128 || plan.bn == 256, "gemm_bf16: bn");
  Params p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.num_m = (M + BM - 1) / BM;
  p.num_n = (N + plan.bn - 1) / plan.bn;
  p.num_kb = (K + BK - 1) / BK;
  p.splits = std::max(1, std::min<int>(plan.splits, p.num_kb));
  p.kb_per_split = (p.num_kb + p.splits - 1) / p.splits;
  p.splits = (p.num_kb + p.kb_per_split - 1) / p.kb_per_split;
  p.total_units = p.num_m * p.num_n * p.splits;
  p.err = a.err;
  p.ldc = (int)a.ldc;

  const CUtensorMap ta = make_tma_2d(const_cast<void*>(a.A), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                     K, M, a.lda, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tb = make_tma_2d(const_cast<void*>(a.B), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                     K, N, a.ldb, BK, plan.bn, CU_TENSOR_MAP_SWIZZLE_128B);

  if (p.splits == 1) {
    p.C = a.C;
    if (a.mode == kModeStore)
      dispatch_bn<kStore>(plan.bn, ta, tb, p, stream);
    else if (a.mode == kModeSiluMul)
      dispatch_bn<kSiluMul>(plan.bn, ta, tb, p, stream);
    else
      dispatch_bn<kF32>(plan.bn, ta, tb, p, stream);
    return;
  }
  const int64_t need = (int64_t)p.splits * M * N;
  B200_REQUIRE(a.workspace != nullptr && a.workspace_numel >= need,
               "gemm_bf16: split-K workspace too small");
  p.C = a.workspace;
  p.ldc = N;
  dispatch_bn<kSplitK>(plan.bn, ta, tb, p, stream);
  const int threads = 256;
  if (silu) {
    const size_t total = (size_t)M * (N / 2);
    const int blocks = (int)std::min<size_t>((total + threads - 1) / threads, 148 * 16);
    splitk_reduce_silu_kernel<false><<<blocks, threads, 0, stream>>>(
        a.workspace, reinterpret_cast<__nv_bfloat16*>(a.C), M, N, (int)a.ldc, p.splits);
  } else {
    const size_t total4 = (size_t)M * N / 4;
    const int blocks = (int)std::min<size_t>((total4 + threads - 1) / threads, 148 * 16);
    if (a.mode == kModeF32)
      splitk_reduce_kernel<true><<<blocks, threads, 0, stream>>>(a.workspace, a.C, M, N,
                                                                 (int)a.ldc, p.splits);
    else
      splitk_reduce_kernel<false><<<blocks, threads, 0, stream>>>(a.workspace, a.C, M, N,
                                                                  (int)a.ldc, p.splits);
  }
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

}  // namespace gemm
}  // namespace b200
