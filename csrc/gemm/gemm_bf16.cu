// Persistent BF16 GEMM on the sm_100a 5th-generation tensor cores.
//
//   C[M, N] = A[M, K] . B[N, K]^T        (A = activations, B = nn.Linear weight, both K-major)
//
// Replaces the vendor BF16 GEMM the reference routes unquantized linears to
// (reference: setup.py:258 links mublasLt; vllm_musa/kernels/fp8_block_gemm.py:18 is its
// Triton GEMM) with a hand-written tcgen05 kernel:
//
//   warp 0      TMA producer: per stage an MT*128 x 64 A tile and a BN x 64 B tile (128-byte
//               swizzle) into a ring of shared-memory slots guarded by full/empty mbarriers.
//   warp 1      allocates TMEM; one elected lane issues tcgen05.mma (M=128, N=BN, K=16; MT
//               of them per k-step, one per 128-row half, all reading the same B tile) and
//               tcgen05.commit.  Accumulators are double-buffered when 2*MT*BN <= 512 columns.
//   warps 2..5  epilogue: tcgen05.ld accumulator rows (16 columns at a time) -> fused
//               epilogue -> global.
//
// BN is a runtime multiple of 16 (16..256) and MT is 1 or 2, so the planner can pick a tile
// count close to a whole number of waves over the 148 SMs (decode-sized M is at the
// compute / bandwidth ridge, where a 1.5-wave tail costs a third of the runtime).  Work units
// (m-tile, n-tile, k-split) are scheduled persistently in grouped order so a wave shares B
// tiles through L2.  Epilogues:
//   kStore     C = acc (bf16)
//   kSiluMul   B rows interleaved in groups of 16 (8 gate rows, 8 up rows); output
//              C[:, g*8 + c] = silu(acc[g*16 + c]) * acc[g*16 + 8 + c]  (N/2 columns)
//   kF32       C = acc (fp32, used for logits)
//   kScatter   C = acc (bf16) stored into the owning rank's receive slot, a peer's memory
//              reached with plain 16-byte stores over NVLink (the reduce-scatter of a
//              row-parallel projection rides on the epilogue; see run_bf16)
// Split-K (any epilogue): units write fp32 partials [splits, M, N]; the CTA that completes an
// output tile last (per-tile arrival counter) sums them and applies the epilogue, so there is
// no separate reduce launch.  Launched with programmatic dependent launch: the producer
// prefetches its first weight tiles into L2, then waits for the previous kernel.
// Every mbarrier wait is bounded (common.cuh); a timeout leaves an error code and the kernel
// drains, frees TMEM and returns.
#include <algorithm>
#include <mutex>
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
constexpr int kMaxStages = 8;
constexpr int kSmemBudget = 226 * 1024;  // dynamic opt-in; leaves room for static smem
constexpr int kSmemOverhead = 1024 /*align*/ + 512 /*barriers, tmem slot*/;
constexpr int kScatterWarpBytes = 32 * 128;  // kScatter epilogue staging per epilogue warp
constexpr int kScatterBytes = 4 * kScatterWarpBytes;

enum Epilogue : int { kStore = 0, kSiluMul = 1, kF32 = 2, kScatter = 3, kStoreT = 4, kSiluT = 5 };

B200_DEVICE void st_cluster_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b),
               "r"(c), "r"(d)
               : "memory");
}

// Transposed ("swap-AB") epilogues compute C^T = W . X^T so a decode-sized token count sits in
// the MMA's N dimension (one 128 x M tile per 128 weight rows, the efficient tcgen05 shape) and
// write C[token][feature] through a per-warp shared-memory transpose.
template <int EPI>
constexpr bool kTransposed = EPI == kStoreT || EPI == kSiluT;

struct Params {
  int M, N, K;
  int bn, stages, acc_bufs, tmem_cols;
  int num_m, num_n, num_kb, splits, kb_per_split;
  int katoms;  // 64-element K atoms per pipeline stage (one TMA box per operand and atom)
  int csplit;  // > 1: split-K over a cluster of csplit CTAs reduced through distributed smem
  int total_units;
  void* C;  // output (bf16 or fp32) or fp32 workspace for split-K
  int ldc;  // elements
  int* err;
  // grouped (MoE) mode: m-tile i uses expert tile_expert[i]'s weights (B rows expert*N ...);
  // the live m-tile count is read from the device (*num_tiles)
  const int32_t* tile_expert;
  const int32_t* num_tiles;
  // split-K: fp32 partials [splits, M, N] and one arrival counter per output tile (zero
  // between launches: the CTA that completes a tile resets it)
  float* ws;
  int* counters;
  // kScatter: receive slots of every rank (peer VAs), rows per owner, this rank
  void* peers[8];
  int rs_rows, rs_rank;
};

B200_DEVICE void epi_barrier() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
B200_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
B200_DEVICE void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
B200_DEVICE void tma_prefetch_l2_2d(const void* desc, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(desc)),
               "r"(x), "r"(y)
               : "memory");
}

B200_HOST_DEVICE int a_tile_bytes(int mt) { return mt * BM * BK * 2; }
B200_HOST_DEVICE int b_tile_bytes(int bn) { return bn * BK * 2; }

B200_DEVICE void unit_coords(int u, const Params& p, int& m, int& n, int& ks) {
  const int tiles = p.num_m * p.num_n;
  int t;
  if (p.csplit > 1) {  // the K splits of a tile are the consecutive CTAs of one cluster
    ks = u % p.csplit;
    t = u / p.csplit;
  } else {
    ks = u / tiles;
    t = u - ks * tiles;
  }
  const int group = kGroupN * p.num_m;
  const int g = t / group;
  const int r = t - g * group;
  const int n0 = g * kGroupN;
  const int gn = min(kGroupN, p.num_n - n0);
  m = r / gn;
  n = n0 + (r - m * gn);
}

B200_DEVICE float silu(float x) { return x / (1.f + __expf(-x)); }

// Transposed store of a 32 x 32 block held one accumulator row per lane: f[j] = C^T(base_row +
// lane, c0 + j).  Writes C[(c0 + lane) * ldc + feature] with 16-byte stores after a shared-
// memory transpose (scr: 2 KB per warp).  kSiluT: rows are gate/up interleaved in groups of 16
// (8 gate rows, then their 8 up rows); the 32-row block yields 16 outputs at base_row / 2.
// Warp-collective: every lane calls it.
template <int EPI>
B200_DEVICE void store_t32(const Params& p, uint8_t* scr, int base_row, int c0,
                           const float (&f)[32], int lane) {
  __nv_bfloat16* s = reinterpret_cast<__nv_bfloat16*>(scr);
  const int t = c0 + lane;
  if constexpr (EPI == kStoreT) {
#pragma unroll
    for (int j = 0; j < 32; ++j) s[j * 32 + lane] = f2bf(f[j]);
    __syncwarp();
    if (t < p.N) {
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.C) + (size_t)t * p.ldc + base_row;
#pragma unroll
      for (int v = 0; v < 4; ++v)
        if (base_row + 8 * v < p.M)
          reinterpret_cast<uint4*>(dst)[v] = reinterpret_cast<const uint4*>(s + lane * 32)[v];
    }
  } else {
    const bool gate = (lane & 8) == 0;
    const int o = (lane & 7) + ((lane >> 4) << 3);  // output index within the block (0..15)
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float up = __shfl_xor_sync(0xffffffffu, f[j], 8);
      if (gate) s[j * 16 + o] = f2bf(silu(f[j]) * up);
    }
    __syncwarp();
    if (t < p.N) {
      __nv_bfloat16* dst =
          reinterpret_cast<__nv_bfloat16*>(p.C) + (size_t)t * p.ldc + base_row / 2;
#pragma unroll
      for (int v = 0; v < 2; ++v)
        if (base_row + 16 * v < p.M)
          reinterpret_cast<uint4*>(dst)[v] = reinterpret_cast<const uint4*>(s + lane * 16)[v];
    }
  }
  __syncwarp();
}

// Final epilogue of 16 accumulator columns [col, col+16) of one row.
template <int EPI>
B200_DEVICE void store_chunk16(const Params& p, int row, int col, const float (&f)[16]) {
  if constexpr (EPI == kSiluMul) {
    // 8 gate columns then the matching 8 up columns -> 8 outputs at col/2
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = silu(f[j]) * f[8 + j];
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.C) + (size_t)row * p.ldc +
                              col / 2) = pack8(o);
  } else if constexpr (EPI == kStore || EPI == kScatter) {
    __nv_bfloat16* C;
    if constexpr (EPI == kScatter) {
      const int owner = row / p.rs_rows;
      C = reinterpret_cast<__nv_bfloat16*>(p.peers[owner]) +
          ((size_t)p.rs_rank * p.rs_rows + (row - owner * p.rs_rows)) * p.ldc + col;
    } else {
      C = reinterpret_cast<__nv_bfloat16*>(p.C) + (size_t)row * p.ldc + col;
    }
#pragma unroll
    for (int v = 0; v < 2; ++v) {
      if (col + 8 * v < p.N) {
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = f[8 * v + j];
        *reinterpret_cast<uint4*>(C + 8 * v) = pack8(o);
      }
    }
  } else {
    float* C = reinterpret_cast<float*>(p.C) + (size_t)row * p.ldc + col;
#pragma unroll
    for (int v = 0; v < 4; ++v)
      if (col + 4 * v < p.N)
        *reinterpret_cast<float4*>(C + 4 * v) =
            make_float4(f[4 * v], f[4 * v + 1], f[4 * v + 2], f[4 * v + 3]);
  }
}

// Cluster split-K reduction (one-CTA kernel, MT = 1).  The csplit CTAs of a cluster computed
// the same 128 x BN tile over different K ranges; each holds its partial sum in TMEM.  Row
// quarter q (TMEM lanes 32q..32q+31, epilogue warp q) is owned by cluster rank q % csplit: the
// other ranks' epilogue warps store their quarter-q rows into the owner's shared memory
// (distributed shared memory, over the idle pipeline ring), and the owner adds them to its own
// rows and runs the epilogue.  Two cluster barriers bracket the exchange; every thread of every
// CTA reaches both, error or not.  Row layout in a receive slot: 32 rows x BN fp32 with the
// 16-byte chunks XOR-swizzled by row (conflict-free 16-byte stores and loads per 8 lanes).
template <int EPI>
B200_DEVICE void csplit_reduce(const Params& p, uint8_t* smem, uint32_t tmem_base, int warp,
                               int lane) {
  const int S = p.csplit;
  const int BN = p.bn;
  const uint32_t rank = cluster_ctarank();
  int m, n, ks;
  unit_coords(blockIdx.x, p, m, n, ks);
  const bool epi = warp >= 2;
  const int q = warp & 3;
  const int owner = q % S;
  const int nch = BN / 4;
  const uint32_t slot_bytes = 32u * BN * 4u;
  const uint32_t region = smem_u32(smem) + (uint32_t)(q / S) * (S - 1) * slot_bytes;
  const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16);
  auto chunk = [&](int c) { return (uint32_t)(((c | 7) < nch ? (c ^ (lane & 7)) : c) * 16); };
  tc::fence_before_sync();
  __syncwarp();
  cluster_sync();  // every accumulator final, every pipeline ring idle
  tc::fence_after_sync();
  if (epi && (int)rank != owner) {
    const int slot = (int)rank < owner ? (int)rank : (int)rank - 1;
    const uint32_t dst = mapa_shared(region + slot * slot_bytes + lane * BN * 4u, owner);
    for (int c = 0; c < BN; c += 16) {
      uint32_t r[16];
      tc::tmem_ld_32x32b_x16(t_row + c, r);
      tc::tmem_ld_wait();
#pragma unroll
      for (int v = 0; v < 4; ++v)
        st_cluster_v4(dst + chunk(c / 4 + v), r[4 * v], r[4 * v + 1], r[4 * v + 2], r[4 * v + 3]);
    }
  }
  __syncwarp();
  cluster_sync();  // every partial delivered
  if (epi && (int)rank == owner) {
    const int row = m * BM + q * 32 + lane;
    const float* mine = reinterpret_cast<const float*>(smem + (region - smem_u32(smem)) +
                                                       lane * BN * 4);
    for (int c = 0; c < BN; c += 16) {
      uint32_t r[16];
      tc::tmem_ld_32x32b_x16(t_row + c, r);
      tc::tmem_ld_wait();
      float f[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) f[j] = __uint_as_float(r[j]);
      for (int sl = 0; sl < S - 1; ++sl) {
        const uint8_t* src = reinterpret_cast<const uint8_t*>(mine) + sl * slot_bytes;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const float4 x = *reinterpret_cast<const float4*>(src + chunk(c / 4 + v));
          f[4 * v] += x.x;
          f[4 * v + 1] += x.y;
          f[4 * v + 2] += x.z;
          f[4 * v + 3] += x.w;
        }
      }
      const int col = n * BN + c;
      if (row < p.M && col < p.N) store_chunk16<EPI>(p, row, col, f);
    }
  }
}

template <int MT, int EPI, bool GROUPED = false>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB, Params p) {
  // Programmatic dependent launch: let the next kernel in the stream start its prologue as
  // soon as SMs free up; it waits (griddepcontrol.wait) before reading what we write.
  pdl_trigger();
  if constexpr (GROUPED) {
    pdl_wait();  // the live tile count is produced by the preceding kernel
    p.num_m = *p.num_tiles;
    p.total_units = p.num_m * p.num_n;
  }
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int STAGES = p.stages;
  const int KA = p.katoms;
  const int A_ATOM = a_tile_bytes(MT);
  const int B_ATOM = b_tile_bytes(p.bn);
  const int A_BYTES = A_ATOM * KA;
  const int B_BYTES = B_ATOM * KA;
  const int STAGE_BYTES = A_BYTES + B_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + kMaxStages;
  uint64_t* acc_full = bars + 2 * kMaxStages;
  uint64_t* acc_empty = bars + 2 * kMaxStages + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kMaxStages + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int BN = p.bn;
  const int ACC_COLS = MT * BN;

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
    tc::tmem_alloc(tmem_slot, p.tmem_cols);
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
      if (!GROUPED && (int)blockIdx.x < p.total_units) {
        // weights do not depend on the previous kernel: start pulling the first unit's B
        // tiles into L2 while that kernel drains
        int m, n, ks;
        unit_coords(blockIdx.x, p, m, n, ks);
        const int kb0 = ks * p.kb_per_split;
        const int kb1 = min(p.num_kb, kb0 + 2 * STAGES);
        for (int kb = kb0; kb < kb1; ++kb)
          for (int a = 0; a < KA; ++a) tma_prefetch_l2_2d(&tmB, (kb * KA + a) * BK, n * BN);
      }
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
          uint8_t* st = smem + stage * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          const int brow = GROUPED ? p.tile_expert[m] * p.N + n * BN : n * BN;
          for (int a = 0; a < KA; ++a) {
            const int x = (kb * KA + a) * BK;
            tma_load_2d(st + a * A_ATOM, &tmA, &full[stage], x, m * BM * MT);
            tma_load_2d(st + A_BYTES + a * B_ATOM, &tmB, &full[stage], x, brow);
          }
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
      const uint32_t idesc = tc::idesc_f16<true>(BM, BN);
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
        const uint32_t d_tmem = tmem_base + acc * ACC_COLS;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          for (int a = 0; a < KA; ++a) {
            const uint64_t bdesc = tc::smem_desc_kmajor_sw128(sa + A_BYTES + a * B_ATOM);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
#pragma unroll
              for (int mt = 0; mt < MT; ++mt) {
                const uint64_t adesc =
                    tc::smem_desc_kmajor_sw128(sa + a * A_ATOM + mt * BM * 128);
                // +32 bytes along K inside the 128-byte swizzle atom -> +2 in the >>4 field
                tc::mma_f16_ss(d_tmem + mt * BN, adesc + 2 * k, bdesc + 2 * k, idesc,
                               (kb > kb0 || a > 0 || k > 0) ? 1u : 0u);
              }
            }
          }
          tc::mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc::mma_commit(&acc_full[acc]);
        if (++acc == p.acc_bufs) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else if (p.csplit > 1) {
    // ------------------------------------------------------------------ cluster split-K
    // one unit per CTA: wait for the accumulator; the exchange follows (csplit_reduce)
    if (mbar_wait(&acc_full[0], 0, p.err)) tc::fence_after_sync();
  } else {
    // ------------------------------------------------------------------ epilogue
    __shared__ int s_last;
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const bool split = p.splits > 1;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = blockIdx.x; u < p.total_units; u += gridDim.x) {
      int m, n, ks;
      unit_coords(u, p, m, n, ks);
      if (!mbar_wait(&acc_full[acc], acc_phase, p.err)) break;
      tc::fence_after_sync();
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int row = (m * MT + mt) * BM + q * 32 + lane;
        const bool row_ok = row < p.M;
        const uint32_t t_row =
            tmem_base + ((uint32_t)(q * 32) << 16) + acc * ACC_COLS + mt * BN;
        if constexpr (kTransposed<EPI>) {
          if (!split) {
            uint8_t* scr = smem + STAGES * STAGE_BYTES + 512 + (warp - 2) * kScatterWarpBytes;
            const int base_row = (m * MT + mt) * BM + q * 32;
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
              const bool two = c + 16 < BN;
              uint32_t r[2][16];
              tc::tmem_ld_32x32b_x16(t_row + c, r[0]);
              if (two) tc::tmem_ld_32x32b_x16(t_row + c + 16, r[1]);
              tc::tmem_ld_wait();
              float f[32];
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                f[j] = __uint_as_float(r[0][j]);
                f[16 + j] = two ? __uint_as_float(r[1][j]) : 0.f;
              }
              store_t32<EPI>(p, scr, base_row, n * BN + c, f, lane);
            }
            continue;
          }
        }
        if constexpr (EPI == kScatter) {
          if (!split) {
            // Stage 32 rows x 64 columns in this warp's scratch, then store each row's 128
            // contiguous bytes with 8 lanes (4 rows per warp instruction): NVLink carries
            // whole 128-byte segments instead of 32-byte row pieces.
            uint8_t* scr = smem + STAGES * STAGE_BYTES + 512 + (warp - 2) * kScatterWarpBytes;
            const int base_row = (m * MT + mt) * BM + q * 32;
#pragma unroll 1
            for (int c = 0; c < BN; c += 64) {
              const int ncol = min(64, BN - c);
              uint32_t r[4][16];
#pragma unroll
              for (int h = 0; h < 4; ++h)
                if (16 * h < ncol) tc::tmem_ld_32x32b_x16(t_row + c + 16 * h, r[h]);
              tc::tmem_ld_wait();
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                if (16 * h >= ncol) continue;
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                  float f[8];
#pragma unroll
                  for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(r[h][8 * j + e]);
                  const int ch = 2 * h + j;
                  *reinterpret_cast<uint4*>(scr + lane * 128 + ((ch ^ (lane & 7)) << 4)) = pack8(f);
                }
              }
              __syncwarp();
              const int chunks = ncol / 8;
              for (int i = lane; i < 32 * chunks; i += 32) {
                const int rl = i / chunks, ch = i - rl * chunks;
                const int rrow = base_row + rl;
                const int col = n * BN + c + ch * 8;
                if (rrow < p.M && col < p.N) {
                  const int owner = rrow / p.rs_rows;
                  __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.peers[owner]) +
                                       ((size_t)p.rs_rank * p.rs_rows + (rrow - owner * p.rs_rows)) *
                                           p.ldc + col;
                  *reinterpret_cast<uint4*>(dst) =
                      *reinterpret_cast<const uint4*>(scr + rl * 128 + ((ch ^ (rl & 7)) << 4));
                }
              }
              __syncwarp();
            }
            continue;
          }
        }
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          const bool two = c + 16 < BN;
          uint32_t r[2][16];
          tc::tmem_ld_32x32b_x16(t_row + c, r[0]);
          if (two) tc::tmem_ld_32x32b_x16(t_row + c + 16, r[1]);
          tc::tmem_ld_wait();
          if (!row_ok) continue;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int col = n * BN + c + 16 * h;
            if ((h == 1 && !two) || col >= p.N) continue;
            if (split) {
              float* w = p.ws + ((size_t)ks * p.M + row) * p.N + col;
#pragma unroll
              for (int v = 0; v < 4; ++v)
                if (col + 4 * v < p.N)  // N % 4 == 0: a float4 is either in or out of the row
                  reinterpret_cast<float4*>(w)[v] = make_float4(
                      __uint_as_float(r[h][4 * v]), __uint_as_float(r[h][4 * v + 1]),
                      __uint_as_float(r[h][4 * v + 2]), __uint_as_float(r[h][4 * v + 3]));
            } else {
              float f[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) f[j] = __uint_as_float(r[h][j]);
              store_chunk16<EPI>(p, row, col, f);
            }
          }
        }
      }
      // accumulator drained: hand TMEM back to the MMA warp
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
      if (++acc == p.acc_bufs) {
        acc = 0;
        acc_phase ^= 1;
      }
      if (split && p.counters != nullptr) {
        // the last CTA to finish this output tile sums the partials and applies the epilogue
        // (no counters: a separate reduction kernel does it after the grid)
        __threadfence();
        epi_barrier();
        const int tile = m * p.num_n + n;
        if (warp == 2 && lane == 0) s_last = atomicAdd(&p.counters[tile], 1) == p.splits - 1;
        epi_barrier();
        if (s_last && kTransposed<EPI>) {
          __threadfence();
          uint8_t* scr = smem + STAGES * STAGE_BYTES + 512 + (warp - 2) * kScatterWarpBytes;
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const int base_row = (m * MT + mt) * BM + q * 32;
            const int row = base_row + lane;
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
              const int col0 = n * BN + c;
              float f[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) f[j] = 0.f;
              if (row < p.M) {
                for (int sp = 0; sp < p.splits; ++sp) {
                  const float* w = p.ws + ((size_t)sp * p.M + row) * p.N + col0;
#pragma unroll
                  for (int v = 0; v < 8; ++v) {
                    if (col0 + 4 * v < p.N && c + 4 * v < BN) {
                      const float4 x = __ldcg(reinterpret_cast<const float4*>(w) + v);
                      f[4 * v] += x.x;
                      f[4 * v + 1] += x.y;
                      f[4 * v + 2] += x.z;
                      f[4 * v + 3] += x.w;
                    }
                  }
                }
              }
              store_t32<EPI>(p, scr, base_row, col0, f, lane);
            }
          }
          epi_barrier();
          if (warp == 2 && lane == 0) p.counters[tile] = 0;
        } else if (s_last) {
          __threadfence();
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const int row = (m * MT + mt) * BM + q * 32 + lane;
            if (row >= p.M) continue;
#pragma unroll 1
            for (int c = 0; c < BN; c += 16) {
              const int col = n * BN + c;
              if (col >= p.N) break;
              float f[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) f[j] = 0.f;
              for (int sp = 0; sp < p.splits; ++sp) {
                const float4* w =
                    reinterpret_cast<const float4*>(p.ws + ((size_t)sp * p.M + row) * p.N + col);
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                  if (col + 4 * v >= p.N) break;
                  const float4 t = __ldcg(w + v);
                  f[4 * v] += t.x;
                  f[4 * v + 1] += t.y;
                  f[4 * v + 2] += t.z;
                  f[4 * v + 3] += t.w;
                }
              }
              store_chunk16<EPI>(p, row, col, f);
            }
          }
          epi_barrier();
          if (warp == 2 && lane == 0) p.counters[tile] = 0;
        }
      }
    }
  }

  if constexpr (!GROUPED && MT == 1 && (EPI == kStore || EPI == kSiluMul || EPI == kF32)) {
    if (p.csplit > 1) csplit_reduce<EPI>(p, smem, tmem_base, warp, lane);
  }
  // peer stores of the scatter epilogue are made visible system-wide before the kernel ends
  if constexpr (EPI == kScatter) __threadfence_system();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 1) tc::tmem_dealloc(tmem_base, p.tmem_cols);
}

// ---------------------------------------------------------------------------------------------
// CTA-pair variant for large M: a 2-CTA cluster computes a 256 x BN tile with cta_group::2
// MMAs.  Each CTA stages its own 128 A rows and half of the BN B rows (same shared-memory
// offsets), so per FLOP the pair moves a third less data from L2 into shared memory than two
// independent 128 x BN tiles.  Both CTAs' TMA loads complete on the leader's full barrier; the
// leader's single MMA thread commits to the empty / accumulator barriers of both CTAs
// (tcgen05.commit multicast); both CTAs' epilogue warps release the accumulator on the
// leader's barrier (8 arrivals).  Split-K as in the one-CTA kernel, per 128-row half tile
// (decode-sized M = 256: one row tile, the K splits fill the SM pairs).
// ---------------------------------------------------------------------------------------------
template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                          const __grid_constant__ CUtensorMap tmB, Params p) {
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int STAGES = p.stages;
  const int BN = p.bn, HALF = BN / 2;
  const int KA = p.katoms;
  const int A_ATOM = BM * BK * 2;
  const int B_ATOM = HALF * BK * 2;
  const int A_BYTES = A_ATOM * KA;
  const int B_BYTES = B_ATOM * KA;
  const int STAGE_BYTES = A_BYTES + B_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + kMaxStages;
  uint64_t* acc_full = bars + 2 * kMaxStages;
  uint64_t* acc_empty = bars + 2 * kMaxStages + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kMaxStages + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const bool leader = crank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 8);  // 4 epilogue warps in each CTA of the pair
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc_pair(tmem_slot, p.tmem_cols);
    tc::tmem_relinquish_pair();
  }
  tc::fence_before_sync();
  cluster_sync();  // both CTAs' barriers and TMEM are ready
  tc::fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      pdl_wait();
      for (int u = pair; u < p.total_units && ok; u += npairs) {
        int m, n, ks;
        unit_coords(u, p, m, n, ks);
        const int kb0 = ks * p.kb_per_split, kb1 = min(p.num_kb, kb0 + p.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + stage * STAGE_BYTES;
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * STAGE_BYTES);
          const uint32_t fullc = mapa_shared(smem_u32(&full[stage]), 0);
          for (int a = 0; a < KA; ++a) {
            const int x = (kb * KA + a) * BK;
            tma_load_2d_pair(st + a * A_ATOM, &tmA, fullc, x, m * 2 * BM + (int)crank * BM);
            tma_load_2d_pair(st + A_BYTES + a * B_ATOM, &tmB, fullc, x,
                             n * BN + (int)crank * HALF);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (ok) {  // no TMA write in flight at exit
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
    if (lane == 0 && leader) {
      const uint32_t idesc = tc::idesc_f16<true>(2 * BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int u = pair; u < p.total_units && ok; u += npairs) {
        int m, n, ks;
        unit_coords(u, p, m, n, ks);
        const int kb0 = ks * p.kb_per_split, kb1 = min(p.num_kb, kb0 + p.kb_per_split);
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, p.err)) break;
        tc::fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          for (int a = 0; a < KA; ++a) {
            const uint64_t adesc = tc::smem_desc_kmajor_sw128(sa + a * A_ATOM);
            const uint64_t bdesc = tc::smem_desc_kmajor_sw128(sa + A_BYTES + a * B_ATOM);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              tc::mma_f16_ss_pair(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc,
                                  (kb > kb0 || a > 0 || k > 0) ? 1u : 0u);
          }
          tc::mma_commit_pair_mc(&empty[stage], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc::mma_commit_pair_mc(&acc_full[acc], 0x3);
        if (++acc == p.acc_bufs) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    __shared__ int s_last;
    const int q = warp & 3;
    const bool split = p.splits > 1;
    const uint32_t acc_empty_leader0 = mapa_shared(smem_u32(&acc_empty[0]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = pair; u < p.total_units; u += npairs) {
      int m, n, ks;
      unit_coords(u, p, m, n, ks);
      if (!mbar_wait(&acc_full[acc], acc_phase, p.err)) break;
      tc::fence_after_sync();
      const int row = m * 2 * BM + (int)crank * BM + q * 32 + lane;
      const bool row_ok = row < p.M;
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        const bool two = c + 16 < BN;
        uint32_t r[2][16];
        tc::tmem_ld_32x32b_x16(t_row + c, r[0]);
        if (two) tc::tmem_ld_32x32b_x16(t_row + c + 16, r[1]);
        tc::tmem_ld_wait();
        if (!row_ok) continue;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int col = n * BN + c + 16 * h;
          if ((h == 1 && !two) || col >= p.N) continue;
          if (split) {
            float* w = p.ws + ((size_t)ks * p.M + row) * p.N + col;
#pragma unroll
            for (int v = 0; v < 4; ++v)
              if (col + 4 * v < p.N)
                reinterpret_cast<float4*>(w)[v] = make_float4(
                    __uint_as_float(r[h][4 * v]), __uint_as_float(r[h][4 * v + 1]),
                    __uint_as_float(r[h][4 * v + 2]), __uint_as_float(r[h][4 * v + 3]));
            continue;
          }
          float f[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) f[j] = __uint_as_float(r[h][j]);
          store_chunk16<EPI>(p, row, col, f);
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(acc_empty_leader0 + acc * (uint32_t)sizeof(uint64_t));
      if (++acc == p.acc_bufs) {
        acc = 0;
        acc_phase ^= 1;
      }
      if (split && p.counters != nullptr) {
        // per 128-row half tile: the last of the K splits to finish sums the partials
        __threadfence();
        epi_barrier();
        const int tile = (m * 2 + (int)crank) * p.num_n + n;
        if (warp == 2 && lane == 0) s_last = atomicAdd(&p.counters[tile], 1) == p.splits - 1;
        epi_barrier();
        if (s_last) {
          __threadfence();
          if (row_ok) {
#pragma unroll 1
            for (int c = 0; c < BN; c += 16) {
              const int col = n * BN + c;
              if (col >= p.N) break;
              float f[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) f[j] = 0.f;
              for (int sp = 0; sp < p.splits; ++sp) {
                const float4* w =
                    reinterpret_cast<const float4*>(p.ws + ((size_t)sp * p.M + row) * p.N + col);
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                  if (col + 4 * v >= p.N) break;
                  const float4 t = __ldcg(w + v);
                  f[4 * v] += t.x;
                  f[4 * v + 1] += t.y;
                  f[4 * v + 2] += t.z;
                  f[4 * v + 3] += t.w;
                }
              }
              store_chunk16<EPI>(p, row, col, f);
            }
          }
          epi_barrier();
          if (warp == 2 && lane == 0) p.counters[tile] = 0;
        }
      }
    }
  }

  tc::fence_before_sync();
  cluster_sync();  // the peer's remote arrivals and TMEM reads are done
  tc::fence_after_sync();
  if (warp == 1) tc::tmem_dealloc_pair(tmem_base, p.tmem_cols);
}

// ---------------------------------------------------------------------------------------------
// Split-K reduction as its own grid (programmatic dependent launch after the GEMM): one thread
// per (row, 16 columns), consecutive threads on consecutive column chunks of a row, so every
// split's partial rows are read with coalesced 16-byte loads; then the GEMM's epilogue.  Used
// where the in-kernel last-arriver fixup would serialise behind one CTA per tile (CTA-pair
// tiles with one unit per CTA).
// ---------------------------------------------------------------------------------------------
template <int EPI>
__global__ void __launch_bounds__(256) splitk_reduce_kernel(Params p) {
  pdl_wait();  // every split's partials are written
  pdl_trigger();
  const int chunks = (p.N + 15) / 16;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)p.M * chunks) return;
  const int row = (int)(idx / chunks), col = (int)(idx % chunks) * 16;
  float f[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) f[j] = 0.f;
  for (int sp = 0; sp < p.splits; ++sp) {
    const float4* w = reinterpret_cast<const float4*>(p.ws + ((size_t)sp * p.M + row) * p.N + col);
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      if (col + 4 * v < p.N) {
        const float4 t = __ldcg(w + v);
        f[4 * v] += t.x;
        f[4 * v + 1] += t.y;
        f[4 * v + 2] += t.z;
        f[4 * v + 3] += t.w;
      }
    }
  }
  store_chunk16<EPI>(p, row, col, f);
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------
struct Plan {
  int mt, bn, splits;
};

// CTA pairs are used from this many rows (B200_GEMM_PAIR_MIN_ROWS; 0 disables)
static int pair_min_rows() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("B200_GEMM_PAIR_MIN_ROWS");
    v = e ? atoi(e) : 2048;
    if (v <= 0) v = 1 << 30;
  }
  return v;
}

// Tile width for CTA pairs: the widest multiple of 32 (<= 256) whose tile count fills the SM
// pairs in whole waves best.
static int pair_bn(int M, int N) {
  const int pairs = std::max(1, num_sms() / 2);
  const int num_m = (M + 2 * BM - 1) / (2 * BM);
  int best = 256;
  double best_eff = 0.0;
  for (int bn = 256; bn >= 128; bn -= 32) {
    const long tiles = (long)num_m * ((N + bn - 1) / bn);
    const long waves = (tiles + pairs - 1) / pairs;
    const double eff = (double)tiles / (double)(waves * pairs) * (bn >= 192 ? 1.0 : 0.93);
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      best = bn;
    }
  }
  return best;
}

// K atoms per pipeline stage.  Measured on B200 with a TMA-only probe (one CTA per SM, tiled
// 128-byte-swizzled boxes, L2-resident source): a stage's mbarrier round trip costs ~250-340
// ns almost regardless of its size, so one CTA pulls 33 / 66 / 132 GB/s with 8 / 16 / 32 KiB
// stages but 190-230 GB/s with 64 KiB stages (the 148 SMs together saturate L2 at ~19 TB/s).
// A decode-sized GEMM streams its whole K range through few stages per CTA, so stages are
// made at least 48 KiB (two or four 64-element K atoms, one TMA box per operand and atom)
// while at least three still fit.  0: automatic; set_katoms() forces a count (tuning).
static int g_katoms = 0;
void set_katoms(int k) { g_katoms = k; }

static int choose_katoms(int stage1, int K, int splits, int budget) {
  auto ok = [&](int ka, int min_stages) {
    return K % (BK * ka) == 0 && budget / (stage1 * ka) >= min_stages && K / (BK * ka) >= splits;
  };
  if (g_katoms > 0) return ok(g_katoms, 2) || g_katoms == 1 ? g_katoms : 1;
  int ka = 1;
  while (ka < 4 && stage1 * ka < 48 * 1024 && ok(2 * ka, 3)) ka *= 2;
  return ka;
}


// Cost model.  A unit's time is the largest of (a) its MMA time, (b) filling shared memory
// with its A and B tiles through L2 at its share of L2 bandwidth (capped per SM), and (c)
// pulling its B tiles (the weights) from HBM at its share of DRAM bandwidth (capped per SM);
// the slowest SM runs ceil(units / SMs) units and the GEMM cannot beat its DRAM bytes at
// full bandwidth.  Split-K adds the fp32 workspace round trip.  Constants are B200 figures
// (~4000 bf16 MAC/clk/SM at ~1.8 GHz under load, ~6.5 TB/s HBM, ~16 TB/s L2).
static double plan_cost(int M, int N, int K, int mt, int bn, int s, int sms) {
  const int num_m = (M + BM * mt - 1) / (BM * mt);
  const int num_n = (N + bn - 1) / bn;
  const int num_kb = (K + BK - 1) / BK;
  const int kps = (num_kb + s - 1) / s;
  const long units = (long)num_m * num_n * s;
  const long per_sm = (units + sms - 1) / sms;
  const long active = std::min<long>(units, sms);
  const double clk = 1.8e9, mac_per_clk = 4000.0;
  const double mma_t = (double)kps * mt * BM * bn * BK / mac_per_clk / clk;
  const double fill_bytes = (double)(mt * BM + bn) * kps * BK * 2;
  const double fill_t = fill_bytes / std::min(1.6e13 / active, 1.2e11);
  const double dram_bytes = (double)bn * kps * BK * 2;
  const double dram_t = dram_bytes / std::min(6.5e12 / active, 9.0e10);
  const double total_bytes = (double)N * K * 2 + (double)M * K * 2 + (double)M * N * 2;
  double t = std::max(per_sm * std::max(mma_t, std::max(fill_t, dram_t)), total_bytes / 6.5e12);
  t += per_sm * 0.6e-6 + 2.0e-6;  // per-unit epilogue / pipeline fill, launch
  if (s > 1) t += (double)M * N * 4 * (s + 1) / 6.0e12 + 3e-6;
  return t;
}

static Plan choose_plan(int M, int N, int K) {
  const int sms = num_sms();
  Plan best{1, 256, 1};
  double best_cost = 1e30;
  const int num_kb = (K + BK - 1) / BK;
  for (int mt = 1; mt <= 2; ++mt) {
    if (mt == 2 && (M <= BM || M > 1024)) continue;  // MT=2 measured slower at large M
    for (int bn = 256; bn >= 16; bn -= 16) {
      if (2 * mt * bn > 512 && M > 1024) continue;  // large M wants double-buffered TMEM
      for (int s = 1; s <= 16; ++s) {
        if (s > 1 && (num_kb + s - 1) / s < 4) break;
        if (s > 1 && (long)s * M * N > (64l << 20)) break;
        const double c = plan_cost(M, N, K, mt, bn, s, sms);
        if (c < best_cost * 0.995) {
          best_cost = c;
          best = {mt, bn, s};
        }
      }
    }
  }
  return best;
}

// Launch with programmatic stream serialization (the kernel calls griddepcontrol.wait before
// touching anything the previous kernel wrote).
template <typename K>
static void launch_pdl(K kern, int grid, int smem, cudaStream_t stream, const CUtensorMap& ta,
                       const CUtensorMap& tb, const Params& p) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, p);
  if (e != cudaSuccess) {
    cudaGetLastError();  // clear the launch error so later launches do not report it
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, reinterpret_cast<const void*>(kern));
    throw std::runtime_error(
        std::string("b200: gemm launch failed: ") + cudaGetErrorString(e) +
        " grid=" + std::to_string(grid) + " smem=" + std::to_string(smem) +
        " max_dyn_smem=" + std::to_string(fa.maxDynamicSharedSizeBytes) +
        " static_smem=" + std::to_string(fa.sharedSizeBytes) + " regs=" +
        std::to_string(fa.numRegs) + " M=" + std::to_string(p.M) + " N=" + std::to_string(p.N) +
        " K=" + std::to_string(p.K) + " bn=" + std::to_string(p.bn) +
        " stages=" + std::to_string(p.stages) + " units=" + std::to_string(p.total_units));
  }
}

template <int MT, int EPI>
static void launch(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p,
                   cudaStream_t stream) {
  auto kern = gemm_bf16_kernel<MT, EPI>;
  ensure_dynamic_smem(reinterpret_cast<const void*>(kern), kSmemBudget);
  const int smem = p.stages * (a_tile_bytes(MT) + b_tile_bytes(p.bn)) * p.katoms +
                   kSmemOverhead + (EPI == kScatter || kTransposed<EPI> ? kScatterBytes : 0);
  const int grid = std::min(p.total_units, num_sms());
  launch_pdl(kern, grid, smem, stream, ta, tb, p);
  count_launch();
}

template <int EPI>
static void launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p,
                        cudaStream_t stream) {
  auto kern = gemm_bf16_pair_kernel<EPI>;
  ensure_dynamic_smem(reinterpret_cast<const void*>(kern), kSmemBudget);
  const int smem = p.stages * (BM * BK * 2 + (p.bn / 2) * BK * 2) * p.katoms + kSmemOverhead;
  const int pairs = std::max(1, std::min(p.total_units, num_sms() / 2));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    throw std::runtime_error(std::string("b200: pair gemm launch failed: ") +
                             cudaGetErrorString(e) + " grid=" + std::to_string(2 * pairs) +
                             " smem=" + std::to_string(smem));
  }
  count_launch();
}

template <int EPI>
static void launch_splitk_reduce(const Params& p, cudaStream_t stream) {
  const long threads = (long)p.M * ((p.N + 15) / 16);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((threads + 255) / 256));
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B200_CUDA_OK(cudaLaunchKernelEx(&cfg, splitk_reduce_kernel<EPI>, p));
  count_launch();
}

// Split-K partials are reduced by the separate grid (measured 1.2-2.5x faster than the in-kernel
// last-arriver fixup at decode sizes: e.g. M=128 N=4096 K=14336 32.7 vs 60.4 us);
// B200_GEMM_SPLITK_REDUCE=0 keeps the in-kernel fixup for one-CTA tiles.  CTA-pair tiles always
// use the grid; swapped (transposed-store) epilogues keep the fixup.
static bool splitk_reduce_kernel_on() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("B200_GEMM_SPLITK_REDUCE");
    v = (e == nullptr || atoi(e) != 0) ? 1 : 0;
  }
  return v == 1;
}

// Plans with mt = 3 run one-CTA 128-row tiles whose K splits form a cluster and are reduced
// through distributed shared memory (csplit_reduce) instead of fp32 partials in global memory
// plus a reduction pass.  Measured on decode shapes: a win with two splits (e.g. M = 256,
// N = K = 4096: 16.7 vs 18.6 us; N = 3584, K = 4096: 16.4 vs 19.7 us), a loss once the clusters
// no longer fit one wave (three or four splits with 100+ tiles), so the tuner chooses it per
// shape and the launcher falls back to the global path when the clusters would not all be
// resident at once.  B200_GEMM_CLUSTER_SPLITK=0 disables it.
static bool cluster_splitk_on() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("B200_GEMM_CLUSTER_SPLITK");
    v = (e == nullptr || atoi(e) != 0) ? 1 : 0;
  }
  return v == 1;
}

// How many clusters of `csplit` one-CTA GEMM blocks with `smem` bytes can be resident at once.
template <int EPI>
static int max_active_clusters(int csplit, int smem) {
  static std::mutex mu;
  static std::vector<std::pair<long, int>> cache;
  const long key = (long)csplit << 32 | (unsigned)smem;
  std::lock_guard<std::mutex> g(mu);
  for (auto& kv : cache)
    if (kv.first == key) return kv.second;
  auto kern = gemm_bf16_kernel<1, EPI>;
  ensure_dynamic_smem(reinterpret_cast<const void*>(kern), kSmemBudget);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(csplit * 64);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = csplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cache.push_back({key, n});
  return n;
}

// Largest receive region one cluster rank needs: its owned row quarters x (csplit - 1) slots of
// 32 rows x bn fp32.
static int csplit_region_bytes(int csplit, int bn) {
  const int owned = (4 + csplit - 1) / csplit;
  return owned * (csplit - 1) * 32 * bn * 4;
}

template <int EPI>
static void launch_csplit(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p,
                          cudaStream_t stream) {
  auto kern = gemm_bf16_kernel<1, EPI>;
  ensure_dynamic_smem(reinterpret_cast<const void*>(kern), kSmemBudget);
  const int smem = p.stages * (a_tile_bytes(1) + b_tile_bytes(p.bn)) * p.katoms + kSmemOverhead;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.total_units);  // one unit per CTA; each tile's splits form a cluster
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.csplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    throw std::runtime_error(std::string("b200: cluster split-K gemm launch failed: ") +
                             cudaGetErrorString(e) + " grid=" + std::to_string(p.total_units) +
                             " cluster=" + std::to_string(p.csplit) +
                             " smem=" + std::to_string(smem));
  }
  count_launch();
}

template <int EPI>
static void dispatch_mt(int mt, const CUtensorMap& ta, const CUtensorMap& tb, const Params& p,
                        cudaStream_t s) {
  if (mt == 2)
    launch<2, EPI>(ta, tb, p, s);
  else
    launch<1, EPI>(ta, tb, p, s);
}

// Grouped (MoE) GEMM: A = expert-sorted rows [max_rows, K] (segments padded to 128 rows),
// B = stacked expert weights [E * N, K]; C = [max_rows, N] (or N/2 with SwiGLU).
void run_grouped_bf16(const GroupedGemmArgs& a, cudaStream_t stream) {
  const int N = a.N, K = a.K;
  B200_REQUIRE(K % 8 == 0 && N % 16 == 0, "grouped gemm: K % 8 == 0 and N % 16 == 0");
  B200_REQUIRE(a.max_rows % BM == 0, "grouped gemm: max_rows must be a multiple of 128");
  if (a.max_rows == 0) return;
  int bn = a.bn > 0 ? a.bn : 0;
  if (bn == 0) {
    // fill the SMs with (tiles x n-tiles) units assuming ~E live tiles
    const int tiles = std::max(1, std::min(a.max_rows / BM, a.num_experts));
    bn = 256;
    while (bn > 64 && (long)tiles * ((N + bn - 1) / bn) < num_sms()) bn -= 64;
  }
  Params p;
  p.M = a.max_rows;
  p.N = N;
  p.K = K;
  p.bn = bn;
  p.csplit = 1;
  {
    const int stage1 = a_tile_bytes(1) + b_tile_bytes(bn);
    const int budget = kSmemBudget - kSmemOverhead;
    p.katoms = choose_katoms(stage1, K, 1, budget);
    p.stages = std::min(kMaxStages, budget / (stage1 * p.katoms));
  }
  p.acc_bufs = 2 * bn <= 512 ? 2 : 1;
  int cols = 32;
  while (cols < p.acc_bufs * bn) cols <<= 1;
  p.tmem_cols = cols;
  p.num_m = a.max_rows / BM;  // upper bound; the kernel reads the live count
  p.num_n = (N + bn - 1) / bn;
  p.num_kb = (K + BK * p.katoms - 1) / (BK * p.katoms);
  p.splits = 1;
  p.kb_per_split = p.num_kb;
  p.total_units = p.num_m * p.num_n;
  p.err = a.err;
  p.ldc = (int)a.ldc;
  p.C = a.C;
  p.tile_expert = a.tile_expert;
  p.num_tiles = a.num_tiles;
  p.ws = nullptr;
  p.counters = nullptr;
  p.rs_rows = p.rs_rank = 0;
  for (int i = 0; i < 8; ++i) p.peers[i] = nullptr;
  const CUtensorMap ta = make_tma_2d(const_cast<void*>(a.A), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                     K, a.max_rows, a.lda, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tb =
      make_tma_2d(const_cast<void*>(a.B), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K,
                  (uint64_t)a.num_experts * N, a.ldb, BK, bn, CU_TENSOR_MAP_SWIZZLE_128B);
  auto go = [&](auto kern) {
    ensure_dynamic_smem(reinterpret_cast<const void*>(kern), kSmemBudget);
    const int smem = p.stages * (a_tile_bytes(1) + b_tile_bytes(bn)) * p.katoms + kSmemOverhead;
    const int grid = std::min(p.total_units, num_sms());
    launch_pdl(kern, grid, smem, stream, ta, tb, p);
  };
  if (a.mode == kModeSiluMul)
    go(gemm_bf16_kernel<1, kSiluMul, true>);
  else
    go(gemm_bf16_kernel<1, kStore, true>);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

GemmPlan plan_bf16(int M, int N, int K) {
  const Plan p = choose_plan(M, N, K);
  const int num_kb = (K + BK - 1) / BK;
  int s = std::max(1, std::min<int>(p.splits, num_kb));
  const int kps = (num_kb + s - 1) / s;
  s = (num_kb + kps - 1) / kps;
  return GemmPlan{p.bn, s, s > 1 ? (int64_t)s * M * N : 0, p.mt};
}

void run_bf16(const GemmArgs& a, cudaStream_t stream) {
  const int M = a.M, N = a.N, K = a.K;
  // (swapped modes: N is the token count, M the weight rows; both must be multiples of 8)
  B200_REQUIRE(K % 8 == 0 && N % 8 == 0, "gemm_bf16: K and N must be multiples of 8");
  B200_REQUIRE((a.mode != kModeStoreT && a.mode != kModeSiluT) || M % 8 == 0,
               "gemm_bf16 swapped: weight rows must be a multiple of 8");
  B200_REQUIRE((a.lda * 2) % 16 == 0 && (a.ldb * 2) % 16 == 0,
               "gemm_bf16: row strides must be 16-byte multiples");
  B200_REQUIRE(reinterpret_cast<uintptr_t>(a.A) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(a.B) % 16 == 0,
               "gemm_bf16: operands must be 16-byte aligned");
  if (M == 0) return;
  const bool silu = a.mode == kModeSiluMul;
  B200_REQUIRE(!silu || N % 16 == 0, "gemm_bf16 silu: N must be a multiple of 16");
  Plan plan = choose_plan(M, N, K);
  if (a.bn > 0) plan.bn = a.bn;
  if (a.splits > 0) plan.splits = a.splits;
  if (a.mt > 0) plan.mt = a.mt;
  // mt = 3: one-CTA tiles (mt 1) with the K splits reduced inside a cluster
  const bool want_cluster = plan.mt == 3;
  if (want_cluster) plan.mt = 1;
  // CTA pairs (mt = 4): 256-row tiles; chosen automatically for large M (no split-K)
  const bool transposed = a.mode == kModeStoreT || a.mode == kModeSiluT;
  B200_REQUIRE(a.mode != kModeSiluT || M % 16 == 0,
               "gemm_bf16 swapped SiLU: weight rows must be a multiple of 16");
  const bool pair_ok = a.mode != kModeScatter && !transposed && M > BM;
  // automatic use (no measured plan): large M and not too wide -- at M = 8192 the pair tiles
  // measured 0.95 / 0.89 of cuBLAS on N = 4096 (K = 14336 / 4096) but lost on N = 28672
  const bool pair = a.mt == 4 ? pair_ok
                              : (a.mt == 0 && a.bn <= 0 && a.splits <= 0 && pair_ok &&
                                 M >= std::max(2 * BM, pair_min_rows()) && N <= 16384 &&
                                 plan.splits <= 1);
  if (!pair && plan.mt == 4) plan.mt = 1;  // a CTA-pair plan for an epilogue pairs lack
  if (pair) {
    plan.mt = 1;
    plan.splits = a.mt == 4 && a.splits > 0 ? a.splits : 1;
    plan.bn = a.mt == 4 && a.bn > 0 && a.bn % 32 == 0 ? a.bn : pair_bn(M, N);
  }
  B200_REQUIRE(plan.bn >= 16 && plan.bn <= 256 && plan.bn % 16 == 0,
               "gemm_bf16: bn must be a multiple of 16 in [16, 256]");
  B200_REQUIRE(plan.mt == 1 || plan.mt == 2,
               "gemm_bf16: mt must be 1, 2, 3 (1 + cluster split-K) or 4 (CTA pair)");
  B200_REQUIRE(!pair || plan.bn % 32 == 0, "gemm_bf16: CTA-pair tiles need bn % 32 == 0");
  Params p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.bn = plan.bn;
  {
    const int stage1 = pair ? BM * BK * 2 + (plan.bn / 2) * BK * 2
                            : a_tile_bytes(plan.mt) + b_tile_bytes(plan.bn);
    // room for the epilogue's shared-memory staging (scatter / transposed stores)
    const int budget = kSmemBudget - kSmemOverhead -
                       (a.mode == kModeScatter || transposed ? kScatterBytes : 0);
    p.katoms = choose_katoms(stage1, K, std::max(1, plan.splits), budget);
    p.stages = std::min(kMaxStages, budget / (stage1 * p.katoms));
  }
  const int acc_cols = plan.mt * plan.bn;
  p.acc_bufs = 2 * acc_cols <= 512 ? 2 : 1;
  B200_REQUIRE(p.stages >= 1, "gemm_bf16: the tile does not fit the shared memory of its CTA");
  int cols = 32;
  while (cols < p.acc_bufs * acc_cols) cols <<= 1;
  p.tmem_cols = cols;
  p.num_m = pair ? (M + 2 * BM - 1) / (2 * BM) : (M + BM * plan.mt - 1) / (BM * plan.mt);
  p.num_n = (N + plan.bn - 1) / plan.bn;
  p.num_kb = (K + BK * p.katoms - 1) / (BK * p.katoms);
  p.splits = std::max(1, std::min<int>(plan.splits, p.num_kb));
  p.kb_per_split = (p.num_kb + p.splits - 1) / p.splits;
  p.splits = (p.num_kb + p.kb_per_split - 1) / p.kb_per_split;
  p.total_units = p.num_m * p.num_n * p.splits;
  p.err = a.err;
  p.ldc = (int)a.ldc;
  p.csplit = 1;
  if (want_cluster && p.splits >= 2 && p.splits <= 4 && cluster_splitk_on() &&
      (a.mode == kModeStore || a.mode == kModeSiluMul || a.mode == kModeF32)) {
    const int ring = p.stages * (a_tile_bytes(1) + b_tile_bytes(plan.bn)) * p.katoms;
    const int smem = ring + kSmemOverhead;
    const int active = a.mode == kModeStore     ? max_active_clusters<kStore>(p.splits, smem)
                       : a.mode == kModeSiluMul ? max_active_clusters<kSiluMul>(p.splits, smem)
                                                : max_active_clusters<kF32>(p.splits, smem);
    if (csplit_region_bytes(p.splits, plan.bn) <= ring && p.num_m * p.num_n <= active)
      p.csplit = p.splits;
  }

  const CUtensorMap ta =
      make_tma_2d(const_cast<void*>(a.A), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, M, a.lda, BK,
                  BM * plan.mt, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tb = make_tma_2d(const_cast<void*>(a.B), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                     K, N, a.ldb, BK, pair ? plan.bn / 2 : plan.bn,
                                     CU_TENSOR_MAP_SWIZZLE_128B);

  p.C = a.C;
  p.tile_expert = nullptr;
  p.num_tiles = nullptr;
  p.ws = nullptr;
  p.counters = nullptr;
  for (int i = 0; i < 8; ++i) p.peers[i] = a.peers[i];
  p.rs_rows = a.rs_rows;
  p.rs_rank = a.rs_rank;
  if (a.mode == kModeScatter) {
    B200_REQUIRE(a.rs_world >= 1 && a.rs_world <= 8 && a.rs_rows > 0 &&
                     (int64_t)a.rs_rows * a.rs_world >= M && a.rs_rank < a.rs_world,
                 "gemm_bf16 scatter: bad reduce-scatter geometry");
    for (int i = 0; i < a.rs_world; ++i)
      B200_REQUIRE(a.peers[i] != nullptr && reinterpret_cast<uintptr_t>(a.peers[i]) % 16 == 0,
                   "gemm_bf16 scatter: receive slots must be 16-byte aligned");
  }
  if (p.splits > 1 && p.csplit == 1) {
    const int64_t need = (int64_t)p.splits * M * N;
    B200_REQUIRE(a.workspace != nullptr && a.workspace_numel >= need,
                 "gemm_bf16: split-K workspace too small");
    B200_REQUIRE(a.counters != nullptr &&
                     a.counters_numel >= (int64_t)p.num_m * p.num_n * (pair ? 2 : 1),
                 "gemm_bf16: split-K tile counters too small");
    p.ws = a.workspace;
    p.counters = a.counters;
  }
  // deferred split-K reduction (separate grid): the GEMM only writes partials
  const bool deferred =
      p.splits > 1 && p.csplit == 1 && (pair || (splitk_reduce_kernel_on() && !transposed));
  if (deferred) p.counters = nullptr;
  if (p.csplit > 1) {
    if (a.mode == kModeStore)
      launch_csplit<kStore>(ta, tb, p, stream);
    else if (a.mode == kModeSiluMul)
      launch_csplit<kSiluMul>(ta, tb, p, stream);
    else
      launch_csplit<kF32>(ta, tb, p, stream);
  } else if (pair) {
    if (a.mode == kModeStore)
      launch_pair<kStore>(ta, tb, p, stream);
    else if (a.mode == kModeSiluMul)
      launch_pair<kSiluMul>(ta, tb, p, stream);
    else
      launch_pair<kF32>(ta, tb, p, stream);
  } else if (a.mode == kModeStore)
    dispatch_mt<kStore>(plan.mt, ta, tb, p, stream);
  else if (a.mode == kModeSiluMul)
    dispatch_mt<kSiluMul>(plan.mt, ta, tb, p, stream);
  else if (a.mode == kModeScatter)
    dispatch_mt<kScatter>(plan.mt, ta, tb, p, stream);
  else if (a.mode == kModeStoreT)
    dispatch_mt<kStoreT>(plan.mt, ta, tb, p, stream);
  else if (a.mode == kModeSiluT)
    dispatch_mt<kSiluT>(plan.mt, ta, tb, p, stream);
  else
    dispatch_mt<kF32>(plan.mt, ta, tb, p, stream);
  if (deferred) {
    if (a.mode == kModeStore)
      launch_splitk_reduce<kStore>(p, stream);
    else if (a.mode == kModeSiluMul)
      launch_splitk_reduce<kSiluMul>(p, stream);
    else if (a.mode == kModeScatter)  // partial sums reduced, then stored into the owners' slots
      launch_splitk_reduce<kScatter>(p, stream);
    else
      launch_splitk_reduce<kF32>(p, stream);
  }
}

}  // namespace gemm
}  // namespace b200
