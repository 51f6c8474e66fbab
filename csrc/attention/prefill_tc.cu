// Causal (chunked) prefill attention on the 5th-generation tensor cores, head_dim 128.
//
// CTA = (128-query tile of one request, one query head); query row i lives in TMEM lane i.
// Warp roles (192 threads, one CTA per SM: 512 TMEM columns, ~162 KB shared memory):
//   warp 0    TMA producer: the Q tile once (two 64-column halves, 128-byte swizzle), then the
//             K and V blocks of 128 keys from the paged cache into two 2-stage rings.
//   warp 1    TMEM owner and single-thread MMA issuer:
//               S_j  = Q K_j^T   M 128, N 128 keys, K 128 dims; Q and K K-major in smem
//               O   += P_j V_j   M 128, N 128 dims, K 128 keys; P from TMEM, V MN-major in smem
//             in the order S_0, S_1, PV_0, S_2, PV_1, ... so the tensor core computes S_{j+1}
//             while the softmax warps work on S_j.
//   warps 2-5 softmax and epilogue, one query row per thread (the TMEM lane quarter its warp
//             may access): tcgen05.ld of the S row, scale + causal / sliding-window mask, online
//             max with lazy rescaling (O is rescaled in TMEM only when a row's running max grows
//             by more than 2^8; until then P = 2^(s - stale max) <= 256), exp2, row sums in
//             registers, P packed to bf16 and written back over the S columns (tcgen05.st).  At
//             the end O / l is read out of TMEM and stored.
// TMEM columns: O [0,128) | S/P buffer 0 [128,256) | 1 [256,384) | 2 [384,512).  With three S
// buffers, S_{j+2} goes to the buffer of P_{j-1}, whose PV has completed by then, so the MMA
// issuer never waits on the MMA it has just issued.
// Every mbarrier wait is bounded (error word + early exit); the producer waits for its own
// copies in flight before the CTA exits, the MMA thread for its MMAs before TMEM is freed.
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
constexpr int kRing = 2;                     // K stages, V stages
constexpr int kTcThreads = 192;
constexpr int kTcSmem = kTileBytes * (1 + 2 * kRing) + 1024 + 256;
constexpr uint32_t kColO = 0, kColS = 128;
constexpr float kRescaleLog2 = 8.f;

struct TcParams {
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

__global__ void tc_tile_offsets_kernel(const int32_t* __restrict__ cu_q, int R,
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
B200_DEVICE void load_kv_block(const CUtensorMap* tm, uint8_t* dst, uint64_t* bar,
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

B200_DEVICE bool warp_wait(uint64_t* bar, uint32_t parity, int* err) {
  const bool ok = mbar_wait(bar, parity, err);
  return __all_sync(0xffffffffu, ok);
}

__global__ void __launch_bounds__(kTcThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                      const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kTileBytes;
  uint8_t* sV = sK + kRing * kTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kRing * kTileBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = bars + 3;
  uint64_t* v_full = bars + 5;
  uint64_t* v_empty = bars + 7;
  uint64_t* s_full = bars + 9;    // [3] S_j computed
  uint64_t* p_full = bars + 12;   // [3] P_j written (4 softmax warps)
  uint64_t* p_free = bars + 15;   // [3] PV_j completed: buffer reusable
  uint64_t* o_done = bars + 18;   // one phase per PV
  uint64_t* fin = bars + 19;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);

  const int tile = p.max_tiles - 1 - blockIdx.x;  // longest-context tiles first
  const int head = blockIdx.y;
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
  const int h = head / (p.Hq / p.Hkv);
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
    for (int b = 0; b < 3; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 4);
      mbar_init(&p_free[b], 1);
    }
    mbar_init(o_done, 1);
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
      mbar_arrive_expect_tx(q_full, kTileBytes);
      tma_load_2d(sQ, &tmQ, q_full, head * kDim, q0);
      tma_load_2d(sQ + kHalfBytes, &tmQ, q_full, head * kDim + 64, q0);
      int nk = 0, nv = 0;  // blocks whose loads were issued
      for (int j = 0; j < nblk; ++j) {
        const int st = j & 1;
        const uint32_t ph = ((j >> 1) & 1) ^ 1;
        if (!mbar_wait(&k_empty[st], ph, p.err)) break;
        load_kv_block(&tmK, sK + st * kTileBytes, &k_full[st], bt, first_blk + j, seq_len, h,
                      p.Hkv, p.block_size);
        ++nk;
        if (!mbar_wait(&v_empty[st], ph, p.err)) break;
        load_kv_block(&tmV, sV + st * kTileBytes, &v_full[st], bt, first_blk + j, seq_len, h,
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
      const uint32_t qa = smem_u32(sQ);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1, b = j % 3;
        if (!mbar_wait(&k_full[st], (j >> 1) & 1, p.err)) return false;
        if (j >= 3 && !mbar_wait(&p_free[b], ((j - 3) / 3) & 1, p.err)) return false;
        tc::fence_after_sync();
        const uint32_t ka = smem_u32(sK + st * kTileBytes);
        const uint32_t d = tmem + kColS + b * 128;
#pragma unroll
        for (int k = 0; k < kDim / 16; ++k) {
          const uint32_t off = (k >> 2) * kHalfBytes;
          tc::mma_f16_ss(d, tc::smem_desc_kmajor_sw128(qa + off) + 2 * (k & 3),
                         tc::smem_desc_kmajor_sw128(ka + off) + 2 * (k & 3), id_s, k > 0);
        }
        tc::mma_commit(&k_empty[st]);
        tc::mma_commit(&s_full[b]);
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int st = j & 1, b = j % 3;
        if (!mbar_wait(&p_full[b], (j / 3) & 1, p.err)) return false;
        if (!mbar_wait(&v_full[st], (j >> 1) & 1, p.err)) return false;
        tc::fence_after_sync();
        const uint32_t va = smem_u32(sV + st * kTileBytes);
        const uint32_t pa = tmem + kColS + b * 128;
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k)  // 16 keys: 8 packed P columns, 16 V rows
          tc::mma_f16_ts(tmem + kColO, pa + 8 * k,
                         tc::smem_desc_mnmajor_sw128(va + k * 16 * 128, kHalfBytes, 1024), id_o,
                         (j > 0 || k > 0) ? 1u : 0u);
        tc::mma_commit(&v_empty[st]);
        tc::mma_commit(&p_free[b]);
        tc::mma_commit(o_done);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, p.err);
      if (ok) ok = issue_s(0);
      if (ok && nblk > 1) ok = issue_s(1);
      for (int j = 0; j < nblk && ok; ++j) {
        ok = issue_pv(j);
        if (ok && j + 2 < nblk) ok = issue_s(j + 2);
      }
      tc::mma_commit(fin);  // every MMA issued above has completed
      mbar_wait(fin, 0, p.err);
    }
  } else {
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    const int my_pos = pos0 + row;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      const int b = j % 3;
      if (!warp_wait(&s_full[b], (j / 3) & 1, p.err)) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      const uint32_t s_col = lane_base + kColS + b * 128;
      uint32_t s[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tc::tmem_ld_32x32b_x32(s_col + 32 * c, s[c]);
      tc::tmem_ld_wait();
      const int kv0 = (first_blk + j) * kBK;
      if (kv0 + kBK - 1 > my_pos || p.window > 0) {  // diagonal / window blocks only
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int kv = kv0 + 32 * c + i;
            if (kv > my_pos || (p.window > 0 && kv <= my_pos - p.window))
              s[c][i] = __float_as_uint(-INFINITY);
          }
      }
      // row max of the raw scores with 8 independent chains (one warp per scheduler: a
      // single dependent chain of 128 max operations would dominate the block)
      float mx8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mx8[k] = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 32; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], __uint_as_float(s[c][i]));
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
      // p = 2^(s * scale - m): one FMA + one ex2 per score, sums in 8 independent chains
      const float neg_m = m_ref == -INFINITY ? 0.f : -m_ref;
      float sum8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) sum8[k] = 0.f;
      uint32_t pk[2][32];
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float a = ex2_approx(fmaf(__uint_as_float(s[c][i]), p.scale_log2, neg_m));
          const float e = ex2_approx(fmaf(__uint_as_float(s[c][i + 1]), p.scale_log2, neg_m));
          sum8[(i >> 1) & 7] += a + e;
          pk[c >> 1][(c & 1) * 16 + i / 2] = pack_bf16x2(a, e);  // low half = even key
        }
#pragma unroll
      for (int k = 0; k < 4; ++k) sum8[k] += sum8[k + 4];
      l += (sum8[0] + sum8[1]) + (sum8[2] + sum8[3]);
      // Every iteration confirms PV_{j-1} (one o_done phase per PV, waited in order: a parity
      // wait is only exact when the barrier is at most one phase ahead of the waiter); O is
      // then stable and may be rescaled before PV_j accumulates into it.
      if (j > 0 && !warp_wait(o_done, (j - 1) & 1, p.err)) {
        ok = false;
        break;
      }
      if (__any_sync(0xffffffffu, resc)) {
        tc::fence_after_sync();
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tc::tmem_ld_32x32b_x32(lane_base + kColO + 32 * c, o);
          tc::tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
          tc::tmem_st_32x32b_x32(lane_base + kColO + 32 * c, o);
        }
      }
      tc::tmem_st_32x32b_x32(s_col, pk[0]);
      tc::tmem_st_32x32b_x32(s_col + 32, pk[1]);
      tc::tmem_st_wait();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[b]);
    }
    if (ok && nblk > 0 && warp_wait(o_done, (nblk - 1) & 1, p.err)) {
      tc::fence_after_sync();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool valid = row < rows;
      __nv_bfloat16* dst = p.o + (int64_t)(q0 + row) * p.ld_o + (int64_t)head * kDim;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tc::tmem_ld_32x32b_x32(lane_base + kColO + 32 * c, o);
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

static int g_prefill_tc = -1;  // -1: read B200_ATTN_TC once

bool prefill_tc_enabled(int D) {
  if (g_prefill_tc < 0) {
    const char* e = getenv("B200_ATTN_TC");
    g_prefill_tc = (e == nullptr || atoi(e) != 0) ? 1 : 0;
  }
  return g_prefill_tc == 1 && D == kDim;
}

void set_prefill_tc(bool on) { g_prefill_tc = on ? 1 : 0; }

void run_prefill_tc(const PrefillArgs& a, cudaStream_t stream) {
  B200_REQUIRE(a.D == kDim, "tensor-core prefill: head_dim must be 128");
  if (prefill_tc2_supported(a.D, a.Hq, a.Hkv)) {
    run_prefill_tc2(a, stream);
    return;
  }
  const int box_rows = a.block_size < 64 ? a.block_size : 64;
  const int64_t cache_rows = (int64_t)a.num_blocks * a.Hkv * a.block_size;
  const CUtensorMap tk = make_tma_2d(a.k_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kDim,
                                     cache_rows, kDim, 64, box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tv = make_tma_2d(a.v_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kDim,
                                     cache_rows, kDim, 64, box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tq = make_tma_2d(const_cast<void*>(a.q), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                     (uint64_t)a.Hq * kDim, a.T, a.ld_q, 64, kBQ,
                                     CU_TENSOR_MAP_SWIZZLE_128B);
  tc_tile_offsets_kernel<<<1, 32, 0, stream>>>(a.cu_q, a.R, a.tile_offsets);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
  TcParams p;
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
  ensure_dynamic_smem(reinterpret_cast<const void*>(prefill_tc_kernel), kTcSmem);
  prefill_tc_kernel<<<dim3(p.max_tiles, a.Hq), kTcThreads, kTcSmem, stream>>>(tq, tk, tv, p);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

}  // namespace attn
}  // namespace b200
