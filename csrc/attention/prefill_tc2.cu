// Causal (chunked) prefill attention on the 5th-generation tensor cores, head_dim 128, two
// query heads of one KV group per CTA.
//
// CTA = (128-query tile of one request, two query heads 2p, 2p+1 that share a KV head); each
// head's 128 query rows live in the TMEM lanes of its own S / O columns.  K and V blocks are
// loaded once and used by both heads (half the K/V shared-memory traffic per FLOP of the
// one-head kernel), and two softmax warpgroups (one per head) give every SM scheduler two
// softmax warps, so one head's exponentials overlap the other head's MMAs.
//   warp 0      TMA producer: Q of both heads once, then K / V blocks of 128 keys (2-stage rings)
//   warp 1      TMEM owner + single-thread MMA issuer, per key block j:
//                 PV0_j, S0_{j+1}, PV1_j, S1_{j+1}   (after S0_0, S1_0)
//               S_h = Q_h K^T (M 128, N 128, K 128); O_h += P_h V (P from TMEM, V MN-major)
//   warps 2-5   softmax + epilogue of head 2p  (thread = query row = TMEM lane)
//   warps 6-9   softmax + epilogue of head 2p+1
// TMEM (512 columns): O0 [0,128) | O1 [128,256) | S0/P0 [256,384) | S1/P1 [384,512).  P_h is
// written over S_h, so S_h(j+1) is issued only after PV_h(j) completed (the MMA thread waits on
// that head's o_done phase); the other head's work keeps the tensor core busy meanwhile.
// Softmax: the S row read with four TMEM loads and one wait, row max in 8 independent chains,
// p = 2^(s*scale - m) with one FMA and one ex2, P packed to bf16 and stored over the S columns
// in 16-column pieces; O rescaled in TMEM
// only when a row max grows by more than 2^8.  Every mbarrier is waited phase by phase (a
// parity wait is exact only while the barrier is at most one phase ahead of the waiter) and
// every wait is bounded (error word + early exit); the producer waits for its own copies in
// flight before exit, the MMA thread for its MMAs before TMEM is freed.
//
// Reference counterpart: the MATE FA3 varlen prefill the reference calls through
// vllm_musa/v1/attention/backends/flash_attn.py:1186-1537 (no kernel source in the reference).
#include <cstdlib>

#include "../b200_kernels.h"
#include "../common/common.cuh"
#include "../common/tcgen05.cuh"
#include "../common/tma_host.h"

namespace b200 {
namespace attn {
namespace {

constexpr int kBQ = 128, kBK = 128, kDim = 128;
constexpr int kHalfBytes = 128 * 128;        // 128 rows x 64 bf16 columns (one swizzle span)
constexpr int kTileBytes = 2 * kHalfBytes;   // 128 rows x 128 columns
constexpr int kRing = 2;
constexpr int kThreads2 = 320;               // 10 warps
// Q0 | Q1 | K ring | V ring | barriers
constexpr int kSmem2 = kTileBytes * (2 + 2 * kRing) + 1024 + 256;
// TMEM columns of head hd's O and S / P
B200_HOST_DEVICE constexpr uint32_t col_o(int hd) { return hd ? 128u : 0u; }
B200_HOST_DEVICE constexpr uint32_t col_s(int hd) { return hd ? 384u : 256u; }
constexpr float kRescaleLog2 = 8.f;

struct Tc2Params {
  __nv_bfloat16* o;
  int64_t ld_o;
  const int32_t* cu_q;
  const int32_t* seq_lens;
  const int32_t* block_tables;
  int64_t bt_stride;
  const int32_t* tile_offsets;  // [R+1], 128-row tiles
  int R, max_tiles, Hq, Hkv, block_size, window;
  float scale_log2;
  int* err;
};

__global__ void tc2_tile_offsets_kernel(const int32_t* __restrict__ cu_q, int R,
                                        int32_t* __restrict__ out) {
  if (threadIdx.x == 0) {
    int acc = 0;
    out[0] = 0;
    for (int r = 0; r < R; ++r) {
      acc += (cu_q[r + 1] - cu_q[r] + kBQ - 1) / kBQ;
      out[r + 1] = acc;
    }
  }
}

// TMA loads of one 128-key block of K or V (kv head h) into a [2 halves][128 rows][128 B] tile.
B200_DEVICE void load_kv_block2(const CUtensorMap* tm, uint8_t* dst, uint64_t* bar,
                                const int32_t* bt, int blk, int n_tok, int h, int Hkv,
                                int block_size) {
  const int box_rows = block_size < 64 ? block_size : 64;
  const int last_page = (n_tok - 1) / block_size;
  mbar_arrive_expect_tx(bar, kTileBytes);
  for (int j = 0; j < kBK / box_rows; ++j) {
    const int tok = blk * kBK + j * box_rows;
    int page = tok / block_size;
    if (page > last_page) page = last_page;  // beyond the sequence: any valid page (masked)
    const int row = (bt[page] * Hkv + h) * block_size + tok % block_size;
    tma_load_2d(dst + j * box_rows * 128, tm, bar, 0, row);
    tma_load_2d(dst + kHalfBytes + j * box_rows * 128, tm, bar, 64, row);
  }
}

B200_DEVICE bool warp_wait2(uint64_t* bar, uint32_t parity, int* err) {
  const bool ok = mbar_wait(bar, parity, err);
  return __all_sync(0xffffffffu, ok);
}

__global__ void __launch_bounds__(kThreads2, 1)
    prefill_tc2_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, Tc2Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;                        // head 0 tile, head 1 tile
  uint8_t* sK = smem + 2 * kTileBytes;       // kRing tiles
  uint8_t* sV = sK + kRing * kTileBytes;     // kRing tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kRing * kTileBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = bars + 3;
  uint64_t* v_full = bars + 5;
  uint64_t* v_empty = bars + 7;
  uint64_t* s_full = bars + 9;    // [head] S_h(j) computed
  uint64_t* p_full = bars + 11;   // [head] P_h(j) written (4 warps)
  uint64_t* o_done = bars + 13;   // [head] PV_h(j) completed
  uint64_t* fin = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int tile = p.max_tiles - 1 - blockIdx.x;  // longest-context tiles first
  const int head0 = 2 * blockIdx.y;
  if (tile >= p.tile_offsets[p.R]) return;
  int lo = 0, hi = p.R - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.tile_offsets[mid] <= tile) lo = mid; else hi = mid - 1;
  }
  const int r = lo;
  const int q_begin = p.cu_q[r], q_end = p.cu_q[r + 1];
  const int q0 = q_begin + (tile - p.tile_offsets[r]) * kBQ;
  const int rows = min(kBQ, q_end - q0);
  const int seq_len = p.seq_lens[r];
  const int pos0 = seq_len - (q_end - q_begin) + (q0 - q_begin);  // position of tile row 0
  const int pos_last = pos0 + rows - 1;
  const int first_blk = p.window > 0 ? max(0, pos0 - p.window + 1) / kBK : 0;
  const int nblk = pos_last / kBK + 1 - first_blk;
  const int h = head0 / (p.Hq / p.Hkv);
  const int32_t* bt = p.block_tables + r * p.bt_stride;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kRing; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int hd = 0; hd < 2; ++hd) {
      mbar_init(&s_full[hd], 1);
      mbar_init(&p_full[hd], 4);
      mbar_init(&o_done[hd], 1);
    }
    mbar_init(fin, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, 2 * kTileBytes);
      for (int hd = 0; hd < 2; ++hd) {
        tma_load_2d(sQ + hd * kTileBytes, &tmQ, q_full, (head0 + hd) * kDim, q0);
        tma_load_2d(sQ + hd * kTileBytes + kHalfBytes, &tmQ, q_full, (head0 + hd) * kDim + 64, q0);
      }
      int nk = 0, nv = 0;  // blocks whose loads were issued
      for (int j = 0; j < nblk; ++j) {
        const int st = j & 1;
        const uint32_t ph = ((j >> 1) & 1) ^ 1;
        if (!mbar_wait(&k_empty[st], ph, p.err)) break;
        load_kv_block2(&tmK, sK + st * kTileBytes, &k_full[st], bt, first_blk + j, seq_len, h,
                       p.Hkv, p.block_size);
        ++nk;
        if (!mbar_wait(&v_empty[st], ph, p.err)) break;
        load_kv_block2(&tmV, sV + st * kTileBytes, &v_full[st], bt, first_blk + j, seq_len, h,
                       p.Hkv, p.block_size);
        ++nv;
      }
      // no copy may still be writing shared memory when the CTA exits
      mbar_wait(q_full, 0, p.err);
      for (int j = nk > kRing ? nk - kRing : 0; j < nk; ++j)
        mbar_wait(&k_full[j & 1], (j >> 1) & 1, p.err);
      for (int j = nv > kRing ? nv - kRing : 0; j < nv; ++j)
        mbar_wait(&v_full[j & 1], (j >> 1) & 1, p.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_s = tc::idesc_f16<true>(kBQ, kBK);
      const uint32_t id_o = tc::idesc_f16<true>(kBQ, kDim) | (1u << 16);  // V is MN-major
      auto issue_s = [&](int hd, int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(&k_full[st], (j >> 1) & 1, p.err)) return false;
        tc::fence_after_sync();
        const uint32_t qa = smem_u32(sQ + hd * kTileBytes);
        const uint32_t ka = smem_u32(sK + st * kTileBytes);
#pragma unroll
        for (int k = 0; k < kDim / 16; ++k) {
          const uint32_t off = (k >> 2) * kHalfBytes;
          tc::mma_f16_ss(tmem + col_s(hd), tc::smem_desc_kmajor_sw128(qa + off) + 2 * (k & 3),
                         tc::smem_desc_kmajor_sw128(ka + off) + 2 * (k & 3), id_s, k > 0);
        }
        tc::mma_commit(&s_full[hd]);
        if (hd == 1) tc::mma_commit(&k_empty[st]);  // both heads' S products read this K
        return true;
      };
      auto issue_pv = [&](int hd, int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(&p_full[hd], j & 1, p.err)) return false;
        if (hd == 0 && !mbar_wait(&v_full[st], (j >> 1) & 1, p.err)) return false;
        tc::fence_after_sync();
        const uint32_t va = smem_u32(sV + st * kTileBytes);
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k)  // 16 keys: 8 packed P columns, 16 V rows
          tc::mma_f16_ts(tmem + col_o(hd), tmem + col_s(hd) + 8 * k,
                         tc::smem_desc_mnmajor_sw128(va + k * 16 * 128, kHalfBytes, 1024), id_o,
                         (j > 0 || k > 0) ? 1u : 0u);
        tc::mma_commit(&o_done[hd]);
        if (hd == 1) tc::mma_commit(&v_empty[st]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, p.err);
      if (ok) ok = issue_s(0, 0) && issue_s(1, 0);
      for (int j = 0; j < nblk && ok; ++j) {
        // S_h(j+1) overwrites P_h(j): it follows that head's PV_h(j) completion.  Head 0's next
        // S is issued before head 1's PV so each head's softmax chain stays short (measured
        // 159.7 us vs 176.7 us with both PVs first, 8 x 1024 tokens, 32 / 8 heads)
        ok = issue_pv(0, j);
        if (ok && j + 1 < nblk) ok = mbar_wait(&o_done[0], j & 1, p.err) && issue_s(0, j + 1);
        if (ok) ok = issue_pv(1, j);
        if (ok && j + 1 < nblk) ok = mbar_wait(&o_done[1], j & 1, p.err) && issue_s(1, j + 1);
      }
      tc::mma_commit(fin);  // every MMA issued above has completed
      mbar_wait(fin, 0, p.err);
    }
  } else {
    const int hd = (warp - 2) >> 2;  // head of this warpgroup
    const int q = warp & 3;          // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    const uint32_t s_col = lane_base + col_s(hd), o_col = lane_base + col_o(hd);
    const int my_pos = pos0 + row;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      if (!warp_wait2(&s_full[hd], j & 1, p.err)) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      const int kv0 = (first_blk + j) * kBK;
      const bool masked = kv0 + kBK - 1 > my_pos || p.window > 0;  // diagonal / window blocks
      // the whole S row in registers: four TMEM loads, one wait
      uint32_t sv[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tc::tmem_ld_32x32b_x32(s_col + 32 * c, sv[c]);
      tc::tmem_ld_wait();
      if (masked) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int kv = kv0 + 32 * c + i;
            if (kv > my_pos || (p.window > 0 && kv <= my_pos - p.window))
              sv[c][i] = __float_as_uint(-INFINITY);
          }
      }
      // row max of the raw scores (8 independent chains)
      float mx8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mx8[k] = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 32; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], __uint_as_float(sv[c][i]));
#pragma unroll
      for (int k = 0; k < 4; ++k) mx8[k] = fmaxf(mx8[k], mx8[k + 4]);
      const float mx = fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])) * p.scale_log2;
      const float m_new = fmaxf(m_ref, mx);
      float factor = 1.f;
      bool resc = false;
      if (m_ref == -INFINITY) {
        m_ref = m_new;  // O holds only zero terms for this row so far
      } else if (m_new > m_ref + kRescaleLog2) {
        factor = ex2_approx(m_ref - m_new);
        resc = true;
        m_ref = m_new;
        l *= factor;
      }
      // p = 2^(s * scale - m) (one FMA + one ex2 per score); P chunk c (16 packed columns)
      const float neg_m = m_ref == -INFINITY ? 0.f : -m_ref;
      float sum8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) sum8[k] = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float a = ex2_approx(fmaf(__uint_as_float(sv[c][i]), p.scale_log2, neg_m));
          const float e = ex2_approx(fmaf(__uint_as_float(sv[c][i + 1]), p.scale_log2, neg_m));
          sum8[(i >> 1) & 7] += a + e;
          pk[i / 2] = pack_bf16x2(a, e);  // low half = even key
        }
        tc::tmem_st_32x32b_x16(s_col + 16 * c, pk);
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) sum8[k] += sum8[k + 4];
      l += (sum8[0] + sum8[1]) + (sum8[2] + sum8[3]);
      // PV_h(j-1) completed (every phase in order); O is stable and may be rescaled
      if (j > 0 && !warp_wait2(&o_done[hd], (j - 1) & 1, p.err)) {
        ok = false;
        break;
      }
      if (__any_sync(0xffffffffu, resc)) {
        tc::fence_after_sync();
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tc::tmem_ld_32x32b_x32(o_col + 32 * c, o);
          tc::tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
          tc::tmem_st_32x32b_x32(o_col + 32 * c, o);
        }
      }
      tc::tmem_st_wait();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[hd]);
    }
    if (ok && warp_wait2(&o_done[hd], (nblk - 1) & 1, p.err)) {
      tc::fence_after_sync();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool valid = row < rows;
      __nv_bfloat16* dst = p.o + (int64_t)(q0 + row) * p.ld_o + (int64_t)(head0 + hd) * kDim;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tc::tmem_ld_32x32b_x32(o_col + 32 * c, o);
        tc::tmem_ld_wait();
        if (!valid) continue;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(o[8 * v + e]) * inv;
          reinterpret_cast<uint4*>(dst + 32 * c)[v] = pack8(f);
        }
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 1) tc::tmem_dealloc(tmem, 512);
}

}  // namespace

static int g_tc2 = -1;  // -1: read B200_ATTN_TC2 once

bool prefill_tc2_supported(int D, int Hq, int Hkv) {
  if (g_tc2 < 0) {
    const char* e = getenv("B200_ATTN_TC2");
    g_tc2 = (e == nullptr || atoi(e) != 0) ? 1 : 0;
  }
  return g_tc2 == 1 && D == kDim && (Hq / Hkv) % 2 == 0;
}

void set_prefill_tc2(bool on) { g_tc2 = on ? 1 : 0; }

void run_prefill_tc2(const PrefillArgs& a, cudaStream_t stream) {
  B200_REQUIRE(a.D == kDim && (a.Hq / a.Hkv) % 2 == 0,
               "two-head tensor-core prefill: head_dim 128 and an even GQA group");
  const int box_rows = a.block_size < 64 ? a.block_size : 64;
  const int64_t cache_rows = (int64_t)a.num_blocks * a.Hkv * a.block_size;
  const CUtensorMap tk = make_tma_2d(a.k_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kDim,
                                     cache_rows, kDim, 64, box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tv = make_tma_2d(a.v_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kDim,
                                     cache_rows, kDim, 64, box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tq = make_tma_2d(const_cast<void*>(a.q), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                     (uint64_t)a.Hq * kDim, a.T, a.ld_q, 64, kBQ,
                                     CU_TENSOR_MAP_SWIZZLE_128B);
  tc2_tile_offsets_kernel<<<1, 32, 0, stream>>>(a.cu_q, a.R, a.tile_offsets);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
  Tc2Params p;
  p.o = reinterpret_cast<__nv_bfloat16*>(a.o);
  p.ld_o = a.ld_o;
  p.cu_q = a.cu_q;
  p.seq_lens = a.seq_lens;
  p.block_tables = a.block_tables;
  p.bt_stride = a.bt_stride;
  p.tile_offsets = a.tile_offsets;
  p.R = a.R;
  p.max_tiles = (a.T + kBQ - 1) / kBQ + a.R;
  p.Hq = a.Hq;
  p.Hkv = a.Hkv;
  p.block_size = a.block_size;
  p.window = a.window;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.err = a.err;
  ensure_dynamic_smem(reinterpret_cast<const void*>(prefill_tc2_kernel), kSmem2);
  prefill_tc2_kernel<<<dim3(p.max_tiles, a.Hq / 2), kThreads2, kSmem2, stream>>>(tq, tk, tv, p);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

}  // namespace attn
}  // namespace b200
